// Beam reorder gather: dst[r] = src[parent[r]] for r < rows, byte-exact.
//
// Rows are `row_bytes` long with their own row strides in src and dst (bytes). This is the
// reference's K/V reorder `kv.index_select(0, parent)` (omniasr_trt/llm.py:237-238, one row =
// one beam's [H, S, D] cache of a layer) and its int32 pointer / token-history reorder
// `ptr.copy_(ptr[parent])`, `hist.copy_(hist[parent])` (omniasr_trt/beam.py:175-176).
//
// An HBM copy: the grid is (row chunks, rows) and every thread moves W-byte words (W = 16 when
// every address, stride and the row length allow it, else 4 or 1) with four loads in flight
// before the stores. A parent outside [0, src_rows) skips its row and sets the status word.

#include "common.cuh"
#include "gather.cuh"

namespace omni {

template <typename W>
__global__ void __launch_bounds__(256) gather_rows_kernel(const GatherArgs a) {
  const int64_t r = blockIdx.y;
  const int64_t p = a.parent64 ? reinterpret_cast<const int64_t*>(a.parent)[r]
                               : (int64_t) reinterpret_cast<const int32_t*>(a.parent)[r];
  if (p < 0 || p >= a.src_rows) {
    if (blockIdx.x == 0 && threadIdx.x == 0) raise_status(a.status, kStatusIndex);
    return;
  }
  const W* s = reinterpret_cast<const W*>(reinterpret_cast<const char*>(a.src) + p * a.src_stride);
  W* d = reinterpret_cast<W*>(reinterpret_cast<char*>(a.dst) + r * a.dst_stride);
  const int64_t n = a.row_bytes / (int64_t)sizeof(W);
  const int64_t step = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * step < n; i += 4 * step) {
    const W x0 = s[i], x1 = s[i + step], x2 = s[i + 2 * step], x3 = s[i + 3 * step];
    d[i] = x0;
    d[i + step] = x1;
    d[i + 2 * step] = x2;
    d[i + 3 * step] = x3;
  }
  for (; i < n; i += step) d[i] = s[i];
}

cudaError_t launch_gather(const GatherArgs& a, int rows, cudaStream_t stream) {
  if (rows <= 0 || a.row_bytes <= 0) return cudaSuccess;
  const uintptr_t bits = (uintptr_t)a.src | (uintptr_t)a.dst | (uintptr_t)a.src_stride |
                         (uintptr_t)a.dst_stride | (uintptr_t)a.row_bytes;
  const int w = (bits % 16 == 0) ? 16 : (bits % 4 == 0) ? 4 : 1;
  const int64_t words = a.row_bytes / w;
  const int64_t per_cta = 256 * 4;
  int64_t chunks = (words + per_cta - 1) / per_cta;
  if (chunks > 65535) chunks = 65535;
  if (chunks < 1) chunks = 1;
  dim3 grid((unsigned)chunks, (unsigned)rows);
  if (w == 16) {
    gather_rows_kernel<uint4><<<grid, 256, 0, stream>>>(a);
  } else if (w == 4) {
    gather_rows_kernel<uint32_t><<<grid, 256, 0, stream>>>(a);
  } else {
    gather_rows_kernel<uint8_t><<<grid, 256, 0, stream>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace omni
