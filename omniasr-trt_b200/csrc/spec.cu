// Speculative decoding's control kernels: the proposal of the next tokens and the acceptance of a drafted step,
// integer work, bit-exact with the reference.
//
// propose: the reference's _propose (omniasr_trt/kernels.py:214-262; PyTorch statement tests/test_spec.py:43-92).
// One CTA per row. Thread i scores draft candidate i (the draft position of the row's newest token at offset
// i - behind from the expected one) and own candidate i (the row's position last-1-i): the number of the row's
// newest `ngram` tokens that precede it, as far as they all match. The best draft candidate has the largest
// score*256 - |offset| among those whose score reaches the `reach` table's need for their distance (leftmost on
// ties); the best own candidate the largest score (the latest on ties). The own tokens win when they match at
// least `self_min` tokens and more than the draft does; they are then continued with their period.
//
// accept: the reference's _accept (kernels.py:264-291). One thread per row: keep argmax 0..n, n being the fed
// tokens' leading run equal to the argmax before them, cut at the first EOS or position >= limit in that run.

#include "common.cuh"
#include "spec.cuh"

namespace omni {

namespace {

// Largest key over the block (all threads get it); keys pack (value, tie order) so the maximum is the winner.
OMNI_DEV uint64_t block_max(uint64_t key, uint64_t* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint64_t other = __shfl_xor_sync(0xffffffffu, key, o);
    key = other > key ? other : key;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red may still be read from a previous call
  if (lane == 0) red[warp] = key;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  uint64_t best = 0;
  for (int w = 0; w < nw; ++w) best = red[w] > best ? red[w] : best;
  return best;
}

__global__ void propose_kernel(const ProposeArgs a) {
  __shared__ int hist[kProposeMaxNgram];
  __shared__ unsigned char hv[kProposeMaxNgram];
  __shared__ uint64_t red[kProposeMaxThreads / 32];
  __shared__ int best_score;
  grid_launch_dependents();
  grid_dependency_wait();  // the token rows and positions come from the kernels before
  const int b = blockIdx.x, i = threadIdx.x;
  const int64_t lst = a.last[b], fst = a.first[b], nx = a.next[b], dl = a.draft_len[b];
  const int32_t* orow = a.out + (int64_t)b * a.s_out;
  const int32_t* drow = a.draft + (int64_t)b * a.s_draft;
  if (lst < 0 || lst >= a.out_cap || fst < 0 || dl < 0 || dl > a.draft_cap) {
    // An index outside its tensor: flag it, propose from the draft at the expected position without reading.
    if (i == 0) {
      raise_status(a.status, kStatusIndex);
      a.use_draft[b] = 1;
      a.start[b] = nx;
    }
    if (i < a.tokens) a.prop[(int64_t)b * a.tokens + i] = 0;
    return;
  }
  if (i < a.ngram) {
    const int64_t hp = lst - i;
    hv[i] = hp >= fst;
    hist[i] = hp >= fst ? orow[hp] : -1;
  }
  __syncthreads();

  // Draft candidate i.
  int rank = -1, score = 0;
  if (i <= a.behind + a.ahead) {
    const int off = i - a.behind;
    const int64_t anchor = nx - 1 + off;
    bool alive = anchor < dl;
    for (int t = 0; t < a.ngram; ++t) {
      const int64_t at = anchor - t;
      alive = alive && at >= 0 && hv[t] && drow[at] == hist[t];
      score += alive;
    }
    const int dist = off < 0 ? -off : off;
    int need = a.ngram;
    for (int r = 3; r >= 0; --r)
      if (dist <= a.reach_dist[r]) need = a.reach_need[r];
    rank = score >= need ? score * 256 - dist : -1;
  }
  const uint64_t dkey = block_max(((uint64_t)(uint32_t)(rank + 1) << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)i), red);
  const int best = (int)(0xFFFFFFFFu - (uint32_t)dkey);
  const bool found = (int)(dkey >> 32) - 1 >= 0;
  if (i == best) best_score = score;

  // Own candidate i: the row's position last - 1 - i.
  int sscore = 0;
  if (i < a.self_slots) {
    const int64_t back = lst - 1 - i;
    bool alive = back >= fst;
    for (int t = 0; t < a.ngram; ++t) {
      const int64_t at = back - t;
      alive = alive && at >= 0 && hv[t] && orow[at] == hist[t];
      sscore += alive;
    }
  }
  const uint64_t skey = block_max(i < a.self_slots ? (((uint64_t)(uint32_t)sscore << 32) |
                                                      (uint32_t)(0xFFFFFFFFu - (uint32_t)i))
                                                   : 0ull,
                                  red);  // its barriers also publish best_score
  const int mine = (int)(skey >> 32);
  const int64_t j = lst - 1 - (int64_t)(0xFFFFFFFFu - (uint32_t)skey);
  const int drafted = found ? best_score : 0;
  const int64_t st = found ? nx + best - a.behind : nx;
  const bool ud = mine < a.self_min || mine <= drafted;
  if (i == 0) {
    a.use_draft[b] = ud;
    a.start[b] = st;
  }
  if (i < a.tokens) {
    int64_t v;
    if (ud) {
      const int64_t at = st + i;
      v = at >= 0 && at < dl ? drow[at] : 0;
    } else {
      const int64_t period = lst - j > 1 ? lst - j : 1;
      v = orow[j + 1 + i % period];
    }
    a.prop[(int64_t)b * a.tokens + i] = v;
  }
}

__global__ void accept_kernel(const AcceptArgs a) {
  grid_launch_dependents();
  grid_dependency_wait();  // the argmax comes from the step's last kernels
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= a.rows || a.done[b]) return;
  const int T = a.width;
  const int64_t p = a.last[b] + 1;
  const int64_t* g = a.argmax + (int64_t)b * T;
  const int64_t* fed = a.tokens + (int64_t)b * T;
  int kept = T - 1;
  for (int j = 0; j + 1 < T; ++j) {
    if (fed[j + 1] != g[j]) {
      kept = j;
      break;
    }
  }
  int n = kept;
  bool ended = false;
  for (int j = 0; j <= kept; ++j) {
    if (g[j] == a.eos || p + j >= a.limit) {
      n = j;
      ended = true;
      break;
    }
  }
  int32_t* orow = a.out + (int64_t)b * a.s_out;
  for (int j = 0; j <= n; ++j) {
    const int64_t at = p + j < a.out_cap ? p + j : a.out_cap - 1;
    if (at < 0) {
      raise_status(a.status, kStatusIndex);
      continue;
    }
    orow[at] = (int32_t)g[j];
  }
  a.tok[b] = g[n];
  a.last[b] = p + n;
  a.done[b] = ended;
  const int64_t base = a.use_draft[b] ? a.start[b] : a.draft_next[b];
  a.draft_next[b] = base + n + 1;
}

}  // namespace

cudaError_t launch_propose(const ProposeArgs& a, int rows, cudaStream_t stream) {
  int slots = a.behind + a.ahead + 1;
  if (a.self_slots > slots) slots = a.self_slots;
  if (a.tokens > slots) slots = a.tokens;
  if (a.ngram > slots) slots = a.ngram;
  const int threads = (slots + 31) / 32 * 32;
  return launch_dependent(propose_kernel, dim3((unsigned)rows), dim3((unsigned)threads), 0, stream, a);
}

cudaError_t launch_accept(const AcceptArgs& a, cudaStream_t stream) {
  const int threads = 128;
  return launch_dependent(accept_kernel, dim3((unsigned)((a.rows + threads - 1) / threads)), dim3(threads), 0,
                          stream, a);
}

}  // namespace omni
