// The generated-key part of beam attention on the tensor-core path (bf16, head_dim 128): row r of a beam step
// attends to its generated keys j < gen_len[r], key j read from cache row ptr[r, j] at position j (the reference's
// _beam_gen, omniasr_trt/kernels.py:115-144). These keys are scattered, a few dozen per row, so the pass is
// latency-bound: one warp per (row, head) issues all of a chunk's loads at once -- lane l scores key l of the chunk
// (its 256-byte K row against the query in shared memory), then accumulates output dims 4l..4l+3 over the chunk's V
// rows -- and all warps of the call run in about one wave. It writes one partial (max, sum, unnormalised output)
// per (row, head), merged with the context segments by combine_tc_kernel. A pointer outside the cache reads the
// row's own cache row and sets the status word's index bit.

#include "attention.cuh"
#include "common.cuh"

namespace omni {

namespace {

constexpr int D = 128;
constexpr int kWarps = 8;

__global__ void __launch_bounds__(kWarps * 32) gen_gather_kernel(const SplitArgs a, int rows) {
  __shared__ float qs[kWarps][D];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t unit = (int64_t)blockIdx.x * kWarps + warp;  // (row, head)
  if (unit >= (int64_t)rows * a.heads) return;
  const int r = (int)(unit / a.heads), h = (int)(unit % a.heads);
  const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(a.q) + unit * D;
  {
    const uint2 u = *reinterpret_cast<const uint2*>(q + 4 * lane);
    qs[warp][4 * lane] = __uint_as_float(u.x << 16);
    qs[warp][4 * lane + 1] = __uint_as_float(u.x & 0xffff0000u);
    qs[warp][4 * lane + 2] = __uint_as_float(u.y << 16);
    qs[warp][4 * lane + 3] = __uint_as_float(u.y & 0xffff0000u);
  }
  __syncwarp();
  int64_t n = a.lengths[r];
  n = n < 0 ? 0 : (n > a.cache_len ? a.cache_len : n);
  const __nv_bfloat16* kb = static_cast<const __nv_bfloat16*>(a.k);
  const __nv_bfloat16* vb = static_cast<const __nv_bfloat16*>(a.v);
  float m = -INFINITY, l = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int64_t j0 = 0; j0 < n; j0 += 32) {
    const int64_t j = j0 + lane;
    const bool valid = j < n;
    int64_t src = r;
    if (valid) {
      const int64_t p = a.ptr[(int64_t)r * a.ptr_stride + j];
      if (p < 0 || p >= a.cache_rows) raise_status(a.status, kStatusIndex);
      else src = p;
    }
    const int64_t off = src * a.s_kb + (int64_t)h * a.s_kh + j * a.s_ks;  // key j's row (elements)
    float s = -INFINITY;
    if (valid) {
      const uint4* kr = reinterpret_cast<const uint4*>(kb + off);
      uint4 w[16];
#pragma unroll
      for (int c = 0; c < 16; ++c) w[c] = kr[c];
      float dot = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const uint32_t x[4] = {w[c].x, w[c].y, w[c].z, w[c].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          dot = fmaf(__uint_as_float(x[e] << 16), qs[warp][8 * c + 2 * e], dot);
          dot = fmaf(__uint_as_float(x[e] & 0xffff0000u), qs[warp][8 * c + 2 * e + 1], dot);
        }
      }
      s = dot * a.qscale;
    }
    float cm = s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
    const float mnew = fmaxf(m, cm);
    const float sc = ex2(m - mnew);  // 0 on the first chunk (m = -inf)
    const float pj = valid ? ex2(s - mnew) : 0.f;
    float ps = pj;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    l = l * sc + ps;
    m = mnew;
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] *= sc;
    // All of the chunk's V loads in flight at once, then the accumulation.
    const int cnt = n - j0 < 32 ? (int)(n - j0) : 32;
    uint2 u[32];
#pragma unroll
    for (int t = 0; t < 32; ++t) {
      const int64_t ot = __shfl_sync(0xffffffffu, off, t);
      u[t] = t < cnt ? *reinterpret_cast<const uint2*>(vb + ot + 4 * lane) : make_uint2(0u, 0u);
    }
#pragma unroll
    for (int t = 0; t < 32; ++t) {
      const float pt = __shfl_sync(0xffffffffu, pj, t);  // 0 past the chunk's keys
      acc[0] = fmaf(pt, __uint_as_float(u[t].x << 16), acc[0]);
      acc[1] = fmaf(pt, __uint_as_float(u[t].x & 0xffff0000u), acc[1]);
      acc[2] = fmaf(pt, __uint_as_float(u[t].y << 16), acc[2]);
      acc[3] = fmaf(pt, __uint_as_float(u[t].y & 0xffff0000u), acc[3]);
    }
  }
  const int64_t part = unit * a.st + a.sp_offset;
  *reinterpret_cast<float4*>(a.part_o + part * D + 4 * lane) = make_float4(acc[0], acc[1], acc[2], acc[3]);
  if (lane == 0) reinterpret_cast<float2*>(a.part_ml)[part] = make_float2(m, l);
}

}  // namespace

cudaError_t launch_gen_gather(const SplitArgs& a, int rows, cudaStream_t stream) {
  const int64_t units = (int64_t)rows * a.heads;
  if (units == 0) return cudaSuccess;
  gen_gather_kernel<<<(unsigned)((units + kWarps - 1) / kWarps), kWarps * 32, 0, stream>>>(a, rows);
  return cudaGetLastError();
}

}  // namespace omni
