#pragma once

#include <stdint.h>

#include <cuda_runtime.h>

namespace omni {

// Causal prefill attention, bf16, head_dim 128 (prefill.cu). Tensors [batch, heads, width, 128] given by base
// pointer and (row, head, position) strides in elements; the head_dim stride is 1.
struct PrefillArgs {
  const void* q;
  int64_t q_sb, q_sh, q_sw;
  const void* k;
  int64_t k_sb, k_sh, k_sw;
  const void* v;
  int64_t v_sb, v_sh, v_sw;
  void* out;
  int64_t o_sb, o_sh, o_sw;
  int batch, heads, width;
  float scale;
  int* status;
};

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream);
// The same for head_dim 512 (prefill_wide.cu): tensors [batch, heads, width, 512].
cudaError_t launch_prefill_wide(const PrefillArgs& a, cudaStream_t stream);

}  // namespace omni
