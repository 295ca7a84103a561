#pragma once

#include <stdint.h>

#include <cuda_runtime.h>

namespace omni {

// One beam-search selection step after the LM head (beam.cu): per group of `beams` rows, the best `beams` of the
// group's beams x vocab candidates, then every row follows its parent (pointer and token-history rows, score,
// count, ended flag) and takes its new token. Row r belongs to group r / beams; the first `groups` groups are
// updated in place. Flags are one byte; per-row and per-group scalars int64 (score fp32).
struct BeamSelectArgs {
  const void* logp;     // [groups * beams, vocab] log-probabilities, bf16 or fp32, row stride s_logp
  int64_t s_logp;
  int logp_f32;         // 1: fp32, 0: bf16
  float* score;         // [rows]
  uint8_t* ended;       // [rows]
  int64_t* count;       // [rows]
  int64_t* tok;         // [rows]
  int32_t* hist;        // [rows, hist_w] stride s_hist
  int64_t s_hist, hist_w;
  int32_t* ptr;         // [rows, ptr_w] stride s_ptr
  int64_t s_ptr, ptr_w;
  int64_t* k_step;      // [groups]
  const int64_t* ctx;   // [groups]
  uint8_t* gdone;       // [groups]
  int groups, beams, vocab, length_norm;
  int64_t eos, pad, limit;
  int* status;
};

constexpr int kBeamSelectMaxBeams = 16;

cudaError_t launch_beam_select(const BeamSelectArgs& a, cudaStream_t stream);

}  // namespace omni
