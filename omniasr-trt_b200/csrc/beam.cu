// Beam search's selection step after the LM head, one CTA per group of beams: the reference's per-group top-k over
// beams x vocab candidates and the reorder of the rows' state by their parents (omniasr_trt/beam.py:161-187),
// exact: the same fp32 operations on the candidates and the same integer updates.
//
// Candidates (beam.py:161-170): cand[b, t] = score[b] + logp[b, t], or with length normalisation, when the group's
// row 0 has counted tokens, (score[b] * count[b] + logp[b, t]) / (count[b] + 1) -- each operation rounded to fp32
// as torch's separate elementwise kernels round it (no contraction); an ended row offers only EOS, at its score.
// The group's best `beams` of its beams x vocab candidates in the order torch.topk(sorted=True) returns them:
// value descending, equal values by flat index ascending. Each thread keeps its own best NB (NB >= beams, a power
// of two) over a strided slice of the candidates; warps merge their lanes' lists, then warp 0 the warps' lists.
//
// Reorder (beam.py:171-187): parent = the winner's beam, new token = its vocabulary index (a group that is done
// keeps every row as it is); ptr and hist rows are copied from the parents' rows (all of a group's parent rows are
// read before any is written, column block by column block), then the row's new token goes into hist at the
// group's step, and score, count, ended, tok, k_step and gdone are updated as the reference updates them.

#include <cooperative_groups.h>

#include "beam.cuh"
#include "common.cuh"

namespace cg = cooperative_groups;

namespace omni {

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kCluster = 8;  // CTAs per group: each scans an eighth of the candidates and copies an eighth of the rows

// A candidate's sort key: a larger key comes first. The value's bits are mapped to an order-preserving unsigned
// integer (-0 counted as +0, every NaN as the largest value, as a comparison-based top-k sees them); the low word
// is the complemented flat index, so equal values order by index ascending. Key 0 is "no candidate".
OMNI_DEV uint64_t cand_key(float v, uint32_t idx) {
  uint32_t b = __float_as_uint(__fadd_rn(v, 0.0f));
  if (v != v) b = 0x7fc00000u;
  const uint32_t o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((uint64_t)o << 32) | (uint32_t)~idx;
}

OMNI_DEV uint32_t key_index(uint64_t key) { return ~(uint32_t)key; }

template <int NB>
OMNI_DEV void insert(uint64_t (&best)[NB], uint64_t key) {
  if (key <= best[NB - 1]) return;
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    if (key > best[j]) {
      const uint64_t t = best[j];
      best[j] = key;
      key = t;
    }
  }
}

OMNI_DEV uint64_t warp_max(uint64_t key) {
  const uint32_t hi = __reduce_max_sync(0xffffffffu, (uint32_t)(key >> 32));
  const uint32_t lo = __reduce_max_sync(0xffffffffu, (uint32_t)(key >> 32) == hi ? (uint32_t)key : 0u);
  return ((uint64_t)hi << 32) | lo;
}

// The warp's best NB keys over its lanes' sorted lists, written by lane 0 to `out`; the lists are consumed.
template <int NB>
OMNI_DEV void warp_merge(uint64_t (&best)[NB], uint64_t* out) {
#pragma unroll
  for (int j = 0; j < NB; ++j) {
    const uint64_t m = warp_max(best[0]);
    if ((threadIdx.x & 31) == 0) out[j] = m;
    if (m != 0 && best[0] == m) {  // keys are unique, so one lane pops its head
#pragma unroll
      for (int i = 0; i + 1 < NB; ++i) best[i] = best[i + 1];
      best[NB - 1] = 0;
    }
  }
}

// The order torch.topk(sorted=True) returns a CUDA tensor's k <= 32 best in (the reference calls it on the group's
// beams x vocab candidates), on the k keys `best` holds in (value descending, index ascending) order: its selection
// lists the values above the k-th best value, then those equal to it, each in index order, and its sort of those k is
// a bitonic network over 32 slots (the unused slots last) that exchanges two entries unless the first is the larger,
// so equal values end up in an order fixed by their slots. One warp, lane = slot; `pre` is 32 words of scratch.
OMNI_DEV void torch_order(uint64_t* best, int n, uint64_t* pre) {
  const int lane = threadIdx.x & 31;
  const uint64_t mine = lane < n ? best[lane] : 0;
  const uint32_t kth = (uint32_t)(best[n - 1] >> 32);
  const bool above = lane < n && (uint32_t)(mine >> 32) > kth;
  const int n_above = __popc(__ballot_sync(0xffffffffu, above));
  int rank = above ? 0 : n_above;  // the place in the selection's list: its class, then index order within it
  for (int i = 0; i < n; ++i) {
    const uint64_t other = __shfl_sync(0xffffffffu, mine, i);
    const bool other_above = (uint32_t)(other >> 32) > kth;
    if (lane < n && other_above == above && key_index(other) < key_index(mine)) ++rank;
  }
  if (lane < n) pre[rank] = mine;
  __syncwarp();
  uint32_t kv = lane < n ? (uint32_t)(pre[lane] >> 32) : 0u;
  uint32_t ix = lane < n ? key_index(pre[lane]) : 0u;
  bool ok = lane < n;
  // One compare-exchange stage: slot `lane` and slot `lane ^ stride`; the lower of the two is the network's first
  // entry, its direction bit `size` of its position (the final merge: always 0).
  auto stage = [&](int size, int stride, bool merge) {
    const uint32_t pk = __shfl_xor_sync(0xffffffffu, kv, stride);
    const uint32_t pi = __shfl_xor_sync(0xffffffffu, ix, stride);
    const bool pv = __shfl_xor_sync(0xffffffffu, ok, stride);
    const bool lower = (lane & stride) == 0;
    const uint32_t ka = lower ? kv : pk, kb = lower ? pk : kv;
    const bool va = lower ? ok : pv, vb = lower ? pv : ok;
    const bool dir = merge ? false : ((lane & ~stride) & size) != 0;
    const bool s = (ka > kb && va) || !vb;
    if (s == dir) {
      kv = pk;
      ix = pi;
      ok = pv;
    }
  };
  for (int size = 2; size < 32; size *= 2)
    for (int stride = size / 2; stride > 0; stride /= 2) stage(size, stride, false);
  for (int stride = 16; stride > 0; stride /= 2) stage(32, stride, true);
  if (lane < n) best[lane] = ((uint64_t)kv << 32) | (uint32_t)~ix;
  __syncwarp();
}

struct Row {
  float score;
  float c, c1;  // count and count + 1 as floats (torch converts the int64 operands to float32)
  int64_t count;
  uint8_t ended;
};

// One candidate's value, as beam.py:163-170 computes it (`norm`: length normalisation on for the group).
OMNI_DEV float cand_value(const BeamSelectArgs& a, const Row& r, bool norm, float lp, int t) {
  if (r.ended) return t == a.eos ? r.score : -INFINITY;
  if (norm) return __fdiv_rn(__fadd_rn(__fmul_rn(r.score, r.c), lp), r.c1);
  return __fadd_rn(r.score, lp);
}

OMNI_DEV float to_float(float x) { return x; }
OMNI_DEV float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }

template <int NB, typename T, int E>
__global__ void __cluster_dims__(kCluster, 1, 1) __launch_bounds__(kThreads) beam_select_kernel(const BeamSelectArgs a) {
  __shared__ Row rows[kBeamSelectMaxBeams];
  __shared__ uint64_t warp_best[kWarps][NB];
  __shared__ uint64_t cta_best[NB];  // read by the other CTAs of the cluster
  __shared__ uint64_t group_best[NB];
  __shared__ int parent_s[kBeamSelectMaxBeams];
  __shared__ uint8_t ended_new[kBeamSelectMaxBeams];

  cg::cluster_group cluster = cg::this_cluster();
  const int q = (int)cluster.block_rank();
  const int g = blockIdx.x / kCluster, n = a.beams, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t row0 = (int64_t)g * n;
  const bool live = a.gdone[g] == 0;
  const int64_t k = a.k_step[g];
  if (tid < n) {
    Row r;
    r.score = a.score[row0 + tid];
    r.count = a.count[row0 + tid];
    r.ended = a.ended[row0 + tid];
    r.c = __ll2float_rn(r.count);
    r.c1 = __ll2float_rn(r.count + 1);
    rows[tid] = r;
  }
  __syncthreads();

  if (live) {
    // ---------------------------------------------------------------- top-k over this CTA's share of the candidates
    const bool norm = a.length_norm && rows[0].count > 0;
    uint64_t best[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) best[j] = 0;
    const int per_row = a.vocab / E;  // E divides vocab on the vector path
    const int total = n * per_row;
    const int share = (total + kCluster - 1) / kCluster;
    const int v0 = q * share, v1 = min(total, v0 + share);
    int b = (v0 + tid) / per_row, t = (v0 + tid - b * per_row) * E;
    for (int vi = v0 + tid; vi < v1; vi += kThreads) {
      const Row r = rows[b];
      const T* src = reinterpret_cast<const T*>(a.logp) + (row0 + b) * a.s_logp + t;
      T vals[E];
      if constexpr (E * sizeof(T) == 16) {
        *reinterpret_cast<uint4*>(vals) = __ldg(reinterpret_cast<const uint4*>(src));
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) vals[e] = src[e];
      }
#pragma unroll
      for (int e = 0; e < E; ++e)
        insert(best, cand_key(cand_value(a, r, norm, to_float(vals[e]), t + e), (uint32_t)(b * a.vocab + t + e)));
      t += kThreads * E;
      while (t >= a.vocab) {
        t -= a.vocab;
        ++b;
      }
    }
    warp_merge(best, warp_best[warp]);
    __syncthreads();
    if (warp == 0) {
#pragma unroll
      for (int j = 0; j < NB; ++j) best[j] = lane < kWarps ? warp_best[lane][j] : 0;
      warp_merge(best, cta_best);
    }
  }
  cluster.sync();  // every CTA's list is complete
  if (live) {
    // Every CTA merges the cluster's lists itself (the same result everywhere), reading the others' shared memory.
    if (warp == 0) {
      uint64_t best[NB];
      const uint64_t* peer = lane < kCluster ? cluster.map_shared_rank(cta_best, lane) : nullptr;
#pragma unroll
      for (int j = 0; j < NB; ++j) best[j] = peer ? peer[j] : 0;
      warp_merge(best, group_best);
    }
  }
  cluster.sync();  // the lists have been read: a CTA may leave once it is done

  if (live && warp == 0) torch_order(group_best, n, warp_best[0]);  // warp_best is free again
  __syncthreads();

  // -------------------------------------------------------------------- parents, new tokens (beam.py:172-178)
  int64_t new_tok = 0;
  float new_score = 0.f;
  int64_t new_count = 0;
  uint8_t new_ended = 0;
  if (tid < n) {
    const int64_t row = row0 + tid;
    int par = tid;
    float top = 0.f;
    if (live) {
      const uint32_t idx = key_index(group_best[tid]);
      par = (int)(idx / (uint32_t)a.vocab);
      const int tv = (int)(idx - (uint32_t)par * (uint32_t)a.vocab);
      new_tok = tv;
      const T* src = reinterpret_cast<const T*>(a.logp) + (row0 + par) * a.s_logp + tv;
      top = cand_value(a, rows[par], a.length_norm && rows[0].count > 0, to_float(*src), tv);
    } else {
      new_tok = a.tok[row];
    }
    const Row p = rows[par];
    if (p.ended) new_tok = a.eos;
    const bool grow = live && !p.ended;
    new_score = grow ? top : p.score;
    new_count = p.count + ((grow && new_tok != a.pad && new_tok != a.eos) ? 1 : 0);
    new_ended = live ? (uint8_t)(new_tok == a.eos) : p.ended;
    parent_s[tid] = par;
    ended_new[tid] = new_ended;
  }
  __syncthreads();

  // -------------------------------------------------------------------- ptr / hist rows follow their parents
  // CTA q of the cluster copies columns [q, q + 1) x width / kCluster of every row: the column ranges are disjoint,
  // so within a range all the group's parent values are read before any is written (one CTA, a barrier between).
  if (live) {
    for (int pass = 0; pass < 2; ++pass) {
      int32_t* base = pass == 0 ? a.ptr : a.hist;
      const int64_t stride = pass == 0 ? a.s_ptr : a.s_hist, width = pass == 0 ? a.ptr_w : a.hist_w;
      const int64_t span = (width + kCluster - 1) / kCluster;
      const int64_t cbeg = q * span, cend = min(width, cbeg + span);
      for (int64_t c0 = cbeg; c0 < cend; c0 += kThreads) {
        const int64_t c = c0 + tid;
        int32_t v[NB];  // n <= NB
#pragma unroll
        for (int j = 0; j < NB; ++j)
          if (j < n && c < cend) v[j] = base[(row0 + parent_s[j]) * stride + c];
        __syncthreads();
#pragma unroll
        for (int j = 0; j < NB; ++j)
          if (j < n && c < cend && parent_s[j] != j) base[(row0 + j) * stride + c] = v[j];
        __syncthreads();
      }
      if (pass == 1 && tid < n) {  // the new token at the group's step, by the CTA whose columns hold it
        if (k >= 0 && k < a.hist_w) {
          if (k >= cbeg && k < cend) a.hist[(row0 + tid) * a.s_hist + k] = (int32_t)new_tok;
        } else if (q == 0) {
          raise_status(a.status, kStatusIndex);
        }
      }
    }
  }

  // -------------------------------------------------------------------- the rows' new state (beam.py:179-187)
  if (q != 0) return;
  if (tid < n) {
    const int64_t row = row0 + tid;
    a.score[row] = new_score;
    a.count[row] = new_count;
    a.ended[row] = new_ended;
    a.tok[row] = new_tok;
  }
  if (tid == 0) {
    bool all_ended = true;
    for (int j = 0; j < n; ++j) all_ended &= ended_new[j] != 0;
    const int64_t ks = k + (live ? 1 : 0);
    a.k_step[g] = ks;
    a.gdone[g] = (uint8_t)(!live || all_ended || (a.ctx[g] - 1 + ks - 1 >= a.limit));
  }
}

template <int NB, typename T>
cudaError_t launch_t(const BeamSelectArgs& a, cudaStream_t stream) {
  constexpr int E = 16 / sizeof(T);
  const bool vec = a.vocab % E == 0 && a.s_logp % E == 0 && reinterpret_cast<uintptr_t>(a.logp) % 16 == 0;
  if (vec)
    beam_select_kernel<NB, T, E><<<a.groups * kCluster, kThreads, 0, stream>>>(a);
  else
    beam_select_kernel<NB, T, 1><<<a.groups * kCluster, kThreads, 0, stream>>>(a);
  return cudaGetLastError();
}

template <int NB>
cudaError_t launch_nb(const BeamSelectArgs& a, cudaStream_t stream) {
  return a.logp_f32 ? launch_t<NB, float>(a, stream) : launch_t<NB, __nv_bfloat16>(a, stream);
}

}  // namespace

cudaError_t launch_beam_select(const BeamSelectArgs& a, cudaStream_t stream) {
  if (a.groups <= 0) return cudaSuccess;
  if (a.beams <= 2) return launch_nb<2>(a, stream);
  if (a.beams <= 4) return launch_nb<4>(a, stream);
  if (a.beams <= 8) return launch_nb<8>(a, stream);
  return launch_nb<16>(a, stream);
}

}  // namespace omni
