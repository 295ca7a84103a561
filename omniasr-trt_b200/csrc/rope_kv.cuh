#pragma once

#include <stdint.h>

#include <cuda_runtime.h>

#include "common.cuh"

namespace omni {

struct RopeArgs {
  const void* qkv;  // [n, 3 * heads * D], unit inner stride
  int64_t qkv_stride;
  const float* cs;  // [cs_positions, D / 2, 2] contiguous
  int64_t cs_positions;
  const int64_t* pos;
  const int64_t* slots;      // may be null: row n
  const int64_t* cache_pos;  // may be null: pos[n]
  void* q_out;               // [n, heads, D] contiguous
  void* k_cache;             // [cache_rows, heads, cache_len, D], strides s_kb, s_kh, s_ks (elements)
  void* v_cache;             // same strides
  int64_t s_kb, s_kh, s_ks, cache_rows, cache_len;
  int heads;
  int* status;
};

// Packs 16 bytes of T from fp32 with round-to-nearest-even.
template <typename T>
struct Pack;

template <>
struct Pack<float> {
  OMNI_DEV static uint4 pack(const float* y) {
    return make_uint4(__float_as_uint(y[0]), __float_as_uint(y[1]), __float_as_uint(y[2]), __float_as_uint(y[3]));
  }
};

template <>
struct Pack<__nv_bfloat16> {
  OMNI_DEV static uint32_t two(float lo, float hi) {
    const uint32_t a = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
    const uint32_t b = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
    return a | (b << 16);
  }
  OMNI_DEV static uint4 pack(const float* y) {
    return make_uint4(two(y[0], y[1]), two(y[2], y[3]), two(y[4], y[5]), two(y[6], y[7]));
  }
};

cudaError_t launch_rope_kv(int dtype, int dim, const RopeArgs& a, int n, cudaStream_t stream);

}  // namespace omni
