// Fused RoPE + KV-cache append.
//
// Token n of `qkv` [N, 3*H*D] (q | k | v) is rotated at position pos[n] with interleaved pairs
// (2j, 2j+1) in fp32, using the caller's table cs [P, D/2, 2] (cos, sin). The rotated q goes to
// q_out [N, H, D]; the rotated k and the raw v are written into the caches at cache row slots[n]
// (default n) and position cache_pos[n] (default pos[n]).
//
// Bit-exactness: the reference rounds each product and the difference separately in fp32
// (omniasr_trt/modeling.py:301-306: re*c - im*s, re*s + im*c, then a round-to-nearest-even cast),
// so this kernel uses non-contracting __fmul_rn / __fsub_rn / __fadd_rn and __float2bfloat16_rn.
// Reference kernel this replaces: omniasr_trt/kernels.py:31-54 (_rope_kv), wrapper :294-306.
//
// Layout: one CTA per (token, section), section 0 = q, 1 = k, 2 = v; each thread moves 16-byte
// vectors. The cs entries of a vector's pairs are the same D-wide row, element for element. Launched as a
// programmatic dependent (launch_dependent), and lets the attention after it start early the same way.

#include "common.cuh"
#include "rope_kv.cuh"

namespace omni {

template <typename T, int D>
__global__ void __launch_bounds__(256) rope_kv_kernel(const RopeArgs a) {
  constexpr int kVec = Elem<T>::kVec;
  constexpr int kPerHead = D / kVec;
  grid_launch_dependents();  // the attention that follows may start its set-up
  grid_dependency_wait();    // qkv, positions and the caches may come from the kernel before
  const int64_t b = blockIdx.x;
  const int part = blockIdx.y;
  const int64_t p = a.pos[b];
  const int64_t row = a.slots ? a.slots[b] : b;
  const int64_t cp = a.cache_pos ? a.cache_pos[b] : p;
  const bool pos_ok = p >= 0 && p < a.cs_positions;
  const bool dst_ok = row >= 0 && row < a.cache_rows && cp >= 0 && cp < a.cache_len;
  if (threadIdx.x == 0 && ((part < 2 && !pos_ok) || !dst_ok)) raise_status(a.status, kStatusIndex);

  const T* src = reinterpret_cast<const T*>(a.qkv) + b * a.qkv_stride + (int64_t)part * a.heads * D;
  const int nvec = a.heads * kPerHead;
  for (int w = threadIdx.x; w < nvec; w += blockDim.x) {
    const int h = w / kPerHead;
    const int c = w - h * kPerHead;
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(src + (int64_t)w * kVec));
    const int64_t cache_off = row * a.s_kb + (int64_t)h * a.s_kh + cp * a.s_ks + c * kVec;
    if (part == 2) {
      if (dst_ok) *reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.v_cache) + cache_off) = u;
      continue;
    }
    uint4 r = make_uint4(0u, 0u, 0u, 0u);
    if (pos_ok) {
      float x[kVec], cs[kVec];
      Elem<T>::unpack(u, x);
      const float4* cr = reinterpret_cast<const float4*>(a.cs + p * D + c * kVec);
#pragma unroll
      for (int i = 0; i < kVec / 4; ++i) {
        const float4 f = __ldg(cr + i);
        cs[4 * i] = f.x;
        cs[4 * i + 1] = f.y;
        cs[4 * i + 2] = f.z;
        cs[4 * i + 3] = f.w;
      }
      float y[kVec];
#pragma unroll
      for (int j = 0; j < kVec / 2; ++j) {
        const float re = x[2 * j], im = x[2 * j + 1];
        const float co = cs[2 * j], si = cs[2 * j + 1];
        y[2 * j] = __fsub_rn(__fmul_rn(re, co), __fmul_rn(im, si));
        y[2 * j + 1] = __fadd_rn(__fmul_rn(re, si), __fmul_rn(im, co));
      }
      r = Pack<T>::pack(y);
    }
    if (part == 0) {
      *reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.q_out) + (b * a.heads + h) * D + c * kVec) = r;
    } else if (dst_ok && pos_ok) {
      *reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.k_cache) + cache_off) = r;
    }
  }
}

template <typename T>
static cudaError_t launch_rope_t(int dim, const RopeArgs& a, int n, cudaStream_t s) {
  dim3 grid((unsigned)n, 3u);
  switch (dim) {
    case 16:
      return launch_dependent(rope_kv_kernel<T, 16>, grid, dim3(256), 0, s, a);
    case 32:
      return launch_dependent(rope_kv_kernel<T, 32>, grid, dim3(256), 0, s, a);
    case 64:
      return launch_dependent(rope_kv_kernel<T, 64>, grid, dim3(256), 0, s, a);
    case 128:
      return launch_dependent(rope_kv_kernel<T, 128>, grid, dim3(256), 0, s, a);
    case 256:
      return launch_dependent(rope_kv_kernel<T, 256>, grid, dim3(256), 0, s, a);
    case 512:
      return launch_dependent(rope_kv_kernel<T, 512>, grid, dim3(256), 0, s, a);
    default:
      return cudaErrorInvalidValue;
  }
}

cudaError_t launch_rope_kv(int dtype, int dim, const RopeArgs& a, int n, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  if (dtype == 0) return launch_rope_t<__nv_bfloat16>(dim, a, n, stream);
  return launch_rope_t<float>(dim, a, n, stream);
}

}  // namespace omni
