#pragma once

#include <stdint.h>

#include <cuda_runtime.h>

namespace omni {

// Speculative decoding's proposal (spec.cu): per row, the next `tokens` proposed tokens from the draft or from the
// row's own tokens. Token rows are int32 (out [rows, out_cap] stride s_out, draft [rows, draft_cap] stride
// s_draft); per-row scalars int64; use_draft one byte per row.
struct ProposeArgs {
  const int32_t* out;
  int64_t s_out, out_cap;
  const int32_t* draft;
  int64_t s_draft, draft_cap;
  const int64_t* draft_len;
  const int64_t* last;
  const int64_t* first;
  const int64_t* next;
  int64_t* start;
  int64_t* prop;       // [rows, tokens]
  uint8_t* use_draft;  // [rows]
  int tokens, ngram, behind, ahead, self_slots, self_min;
  int reach_dist[4], reach_need[4];
  int* status;
};

// After a drafted step: keep the fed tokens equal to the argmax before them (spec.cu).
struct AcceptArgs {
  const int64_t* tokens;  // [rows, width]: the newest token, then the proposal
  const int64_t* argmax;  // [rows, width]
  int32_t* out;
  int64_t s_out, out_cap;
  int64_t* tok;
  int64_t* last;
  uint8_t* done;
  int64_t* draft_next;
  const int64_t* start;
  const uint8_t* use_draft;
  int rows, width;
  int64_t limit, eos;
  int* status;
};

constexpr int kProposeMaxThreads = 1024;
constexpr int kProposeMaxNgram = 32;

cudaError_t launch_propose(const ProposeArgs& a, int rows, cudaStream_t stream);
cudaError_t launch_accept(const AcceptArgs& a, cudaStream_t stream);

}  // namespace omni
