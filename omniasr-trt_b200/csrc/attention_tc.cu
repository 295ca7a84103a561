// Split-KV attention over a bf16 KV cache on the 5th-generation tensor cores (tcgen05 + TMEM), head_dim 128,
// up to 16 queries per group (decode: 1, draft verify: 1 + k, beam context: beams).
//
// Schedule (persistent, stream-K): the keys of every (group, head) unit are cut into 128-key tiles; the grid is
// one CTA per SM and CTA b takes the contiguous tile range [b * per, (b + 1) * per) of the concatenated units, so
// every SM streams the same number of K/V bytes whatever the ragged lengths. A unit cut between CTAs leaves one
// partial (max, sum, unnormalised output) per CTA ("segment"). For decode and draft calls the last CTA to finish a
// unit merges its segments itself (a per-unit counter at the head of the workspace says which CTA is last); for
// beam search, whose generated keys are attended separately, a combine kernel merges them.
//
// One CTA (256 threads): warp 4 loads the queries and the K tiles, warp 6 the V tiles (TMA, two 64-column boxes
// each, 128-byte swizzle, three 32 KB slots per operand); warp 5 issues the MMAs; warps 0-3 run the softmax,
// thread t owning TMEM lane t; warp 7 writes finished units out:
//   S^T[128 keys x 16 q]  = K_tile [128 x 128] . Q^T         (tcgen05.mma, M=128 N=16, K-major A and B)
//   softmax over the keys of each query column (online, fp32, log2 units), P^T written to shared memory (bf16)
//   O^T[128 dims x 16 q]  = V_tile^T [128 x 128 keys] . P^T   (M=128 N=16, MN-major A and B)
// The per-tile O^T is read back from TMEM one tile later and accumulated in registers (thread t = head dim t);
// a unit's accumulator goes through a shared-memory stash to warp 7, so a unit boundary costs the softmax warps
// no global stores. The set-up before griddepcontrol.wait overlaps the previous kernel (programmatic launch).
//
// Algorithm of the reference restated: omniasr_trt/kernels.py:56-113 (_beam_ctx, CAUSAL for drafts) and
// kernels.py:163-195 (_attn_split): the same online softmax per split, merged by the combine
// (kernels.py:146-161 / :197-211).

#include <cudaTypedefs.h>

#include <algorithm>
#include <math.h>
#include <stdlib.h>

#include "attention.cuh"
#include "tc.cuh"

#include "trace.cuh"

namespace omni {

namespace tcattn {

constexpr int D = 128;
constexpr int BN = 128;          // keys per tile (the MMA's M)
constexpr int NQP = 16;          // query columns (the MMA's N)
constexpr int SLOT_BYTES = BN * D * 2;  // one K or V tile
constexpr int BOX_BYTES = BN * 64 * 2;  // one 64-column box of a tile

// Shared-memory layout of a CTA with SLOTS tile slots: K of tile i in slot i % (SLOTS / 2), V in slot
// SLOTS / 2 + i % (SLOTS / 2), so K loads never wait behind V loads (each has its own producer).
template <int SLOTS, int DIM>
struct Smem {
  static constexpr int Q_OFF = SLOTS * SLOT_BYTES;      // two query buffers (units u and u + 1), NQP x DIM each
  static constexpr int P_OFF = Q_OFF + 2 * NQP * DIM * 2;
  static constexpr int RED_OFF = P_OFF + 2 * NQP * BN * 2;         // column maxima of the 4 softmax warps
  static constexpr int RED_L_OFF = RED_OFF + 4 * NQP * 4;           // column sums of a finished unit
  static constexpr int STASH_M_OFF = RED_L_OFF + 4 * NQP * 4;       // its running max per column
  static constexpr int STASH_OFF = STASH_M_OFF + NQP * 4;           // its accumulator [NQP][DIM dims]
  static constexpr int BYTES = STASH_OFF + NQP * DIM * 4 + 1024;    // + alignment slack
};
// Warps 0-3 softmax, 4 K + query loads, 5 MMA issuer, 6 V loads, 7 write-out; with head_dim 512 also warp 8, which
// zeroes the V rows past a unit's keys in its last tile (the key tile's four 128-dim chunks stream through the ring,
// so the softmax warps, which did this for head_dim 128, cannot wait for all of them).
// With split issue the O^T MMAs have their own issuing thread (the last warp), so that the S^T MMAs of later tiles
// never wait behind the V chunks of an earlier one: head_dim 512, and head_dim 128 up to OMNI_TC_SPLIT_NQ queries per
// unit (measured at head_dim 128, three runs each on one box: decode 4804 -> 4869 GB/s with one query; verify, 8
// query columns, 4232 -> 3968).
#ifndef OMNI_TC_SPLIT_NQ
#define OMNI_TC_SPLIT_NQ 2
#endif
constexpr bool split_issue(int dim, int nqt) { return dim == 512 || nqt <= OMNI_TC_SPLIT_NQ; }
constexpr int pv_warp(int dim) { return dim == 128 ? 8 : 9; }
constexpr int threads_for(int dim, int nqt) {
  return 32 * (split_issue(dim, nqt) ? pv_warp(dim) + 1 : (dim == 128 ? 8 : 9));
}
// TMEM: S^T x2 (cols 0-31), then O^T x2 per 128-dim chunk of the head (16 columns each).
constexpr uint32_t tmem_cols(int dim) { return dim == 128 ? 64u : 256u; }
OMNI_DEV uint32_t ocol(int buf, int chunk, int dc) { return 2 * NQP + (buf * dc + chunk) * NQP; }
constexpr uint32_t IDESC_S = idesc_bf16(128, NQP, 0, 0);
constexpr uint32_t IDESC_O = idesc_bf16(128, NQP, 1, 1);

using Params = TcParams;

// Group g's length: lengths[g], or in prefill mode (a row's queries as groups of nq consecutive positions, kv_div
// groups per cache row) the keys its first query sees, (g % kv_div) * nq + 1.
OMNI_DEV int64_t group_len(const Params& p, int g) {
  return p.prefill ? (int64_t)(g % p.kv_div) * p.nq + 1 : p.lengths[g];
}

// Index of segment s of query row j of unit (g, h) in the partial arrays. In prefill mode only the units cut between
// CTAs have partials, and each CTA is the first CTA of at most one of them: the slot is that CTA's (seg0).
OMNI_DEV int64_t part_index(const Params& p, int g, int j, int h, int s, int64_t seg0) {
  return p.prefill ? (seg0 * p.st + s) * NQP + j : (((int64_t)g * p.nq + j) * p.heads + h) * p.st + s;
}

// Keys unit (g, .) must read, clamped to the cache and the key bound.
OMNI_DEV int64_t unit_need(const Params& p, int g) {
  int64_t n = group_len(p, g) + (p.causal ? p.nq - 1 : 0);
  n = n < 0 ? 0 : n;
  return n > p.cap ? p.cap : n;
}

// Work is split between CTAs by cost, not by tiles: a unit (group, head) costs p.unit_cost for its start and
// epilogue plus kTileCost per tile, and tile t of unit (g, h) sits at cost position
//   pre(g) + h * ucost(g) + unit_cost + kTileCost * t,   pre(g) = sum over earlier groups of heads * ucost.
// CTA b owns the tiles whose position lies in [b * per, (b + 1) * per), per = ceil(total cost / grid).
constexpr int64_t kTileCost = 8;
#ifndef OMNI_TC_L2_PROMOTION
#define OMNI_TC_L2_PROMOTION CU_TENSOR_MAP_L2_PROMOTION_L2_256B  // L2 fill granularity of the K/V boxes
#endif
constexpr int kSmemGroups = 256;  // groups whose lengths the pass keeps in shared memory

OMNI_DEV int64_t unit_cost(const Params& p, int64_t tiles) { return tiles > 0 ? p.unit_cost + kTileCost * tiles : 0; }

OMNI_DEV int64_t total_cost(const Params& p) {
  int64_t c = 0;
  for (int g = 0; g < p.groups; ++g) c += unit_cost(p, (unit_need(p, g) + BN - 1) / BN) * p.heads;
  return c;
}

// The tiles of one CTA, in order (groups outer, heads inner, tiles of a unit innermost).
struct TileIter {
  const Params* p;
  int64_t c1;
  int g, h, t;
  int64_t pre, tiles, ucost, need, pos;
  bool done;
  OMNI_DEV void load_group() {
    need = unit_need(*p, g);
    tiles = (need + BN - 1) / BN;
    ucost = unit_cost(*p, tiles);
  }
  // Skips heads past the last and groups without tiles.
  OMNI_DEV void normalize() {
    while (!done && (tiles == 0 || h >= p->heads)) {
      if (g >= p->groups - 1) {
        done = true;
        return;
      }
      pre += ucost * p->heads;
      ++g;
      load_group();
      h = 0;
      t = 0;
    }
  }
  OMNI_DEV void place() {
    if (done) return;
    pos = pre + h * ucost + p->unit_cost + kTileCost * t;
    if (pos >= c1) done = true;
  }
  // pre_tab (optional): pre_tab[g] = cost of the groups before g, for g <= groups (a binary search instead of a
  // walk over the groups).
  OMNI_DEV void init(const Params& pp, int64_t c0, int64_t c1_, const int64_t* pre_tab = nullptr) {
    p = &pp;
    c1 = c1_;
    g = 0;
    pre = 0;
    h = t = 0;
    done = false;
    if (pre_tab) {
      int lo = 0, hi = p->groups - 1;  // the first group that ends past c0 (else the last)
      while (lo < hi) {
        const int mid = (lo + hi) >> 1;
        if (pre_tab[mid + 1] > c0) hi = mid;
        else lo = mid + 1;
      }
      g = lo;
      pre = pre_tab[g];
    }
    load_group();
    while (g < p->groups - 1 && c0 >= pre + ucost * p->heads) {
      pre += ucost * p->heads;
      ++g;
      load_group();
    }
    if (ucost > 0) {
      const int64_t r = c0 - pre;
      h = (int)(r / ucost);
      const int64_t q = r - h * ucost;
      t = q <= p->unit_cost ? 0 : (int)((q - p->unit_cost + kTileCost - 1) / kTileCost);
      if (t >= tiles) {
        t = 0;
        ++h;
      }
    }
    normalize();
    place();
  }
  OMNI_DEV void advance() {
    if (++t >= tiles) {
      t = 0;
      ++h;
    }
    normalize();
    place();
  }
  OMNI_DEV bool last_here() const { return t == tiles - 1 || pos + kTileCost >= c1; }
  OMNI_DEV int64_t unit_pos0() const { return pre + h * ucost + p->unit_cost; }
};

OMNI_DEV bool named_sync_and(int id, int count, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}

// Per-column totals of N values held by each of 32 lanes, in N - 1 + (5 - log2 N) shuffles instead of 5 N:
// each step a lane keeps half of its columns and adds its partner's copy of them. Returns this lane's column
// total and sets `col`; lanes whose low 5 - log2 N bits are zero hold distinct columns.
template <int N, bool MAX>
OMNI_DEV float butterfly(const float (&v)[N], int lane, int& col) {
  float w[N];
#pragma unroll
  for (int i = 0; i < N; ++i) w[i] = v[i];
  int off = 16;
  col = 0;
#pragma unroll
  for (int step = 0; (1 << step) < N; ++step) {
    const int half = N >> (step + 1);
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = upper ? w[i] : w[half + i];
      const float keep = upper ? w[half + i] : w[i];
      const float got = __shfl_xor_sync(0xffffffffu, send, off);
      w[i] = MAX ? fmaxf(keep, got) : keep + got;
    }
    if (upper) col += half;
    off >>= 1;
  }
  float r = w[0];
  for (; off > 0; off >>= 1) {
    const float got = __shfl_xor_sync(0xffffffffu, r, off);
    r = MAX ? fmaxf(r, got) : r + got;
  }
  return r;
}

template <int N>
OMNI_DEV bool butterfly_writer(int lane) {
  return (lane & (32 / N - 1)) == 0;
}

constexpr float kRescale = 8.f;  // log2 units: probabilities may reach 2^8 before the running max is raised
constexpr float kBelow = 64.f;   // ... and the first tile's scores may lie 2^64 below the initial guess

OMNI_DEV bool named_sync_or(int id, int count, bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "barrier.cta.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return out != 0;
}

OMNI_DEV unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Four output dims a * inv as bf16.
OMNI_DEV void store_out4(__nv_bfloat16* dst, const float4& a, float inv) {
  const __nv_bfloat162 lo = __floats2bfloat162_rn(a.x * inv, a.y * inv);
  const __nv_bfloat162 hi = __floats2bfloat162_rn(a.z * inv, a.w * inv);
  uint2 w;
  w.x = *reinterpret_cast<const uint32_t*>(&lo);
  w.y = *reinterpret_cast<const uint32_t*>(&hi);
  *reinterpret_cast<uint2*>(dst) = w;
}

// Output rows of unit (g, h) from its nseg segments: segment `own` from this CTA's stash, the others' from the
// partial arrays (read through L2: other CTAs wrote them). One warp; lane l holds dims 4l .. 4l+3 of each 128-dim
// chunk of the head. Segments go outermost so that a chunk of queries has all its loads of one segment in flight at
// once; the merge is the combine's: out = sum_s w_s o_s / sum_s w_s l_s, w_s = 2^(m_s - max), segments that saw no
// key take no part.
template <int NQT, int DIM>
OMNI_DEV void merge_unit(const Params& p, int g, int h, int own, int nseg, int64_t seg0, int lane, const float* red_l,
                         const float* stash_m, const float* stash) {
  constexpr int DC = DIM / D;
  constexpr int JC = (NQT < 8 ? NQT : 8) / DC > 0 ? (NQT < 8 ? NQT : 8) / DC : 1;  // queries per chunk (registers)
  const float2* ml = reinterpret_cast<const float2*>(p.part_ml);
#pragma unroll 1
  for (int j0 = 0; j0 < NQT && j0 < p.nq; j0 += JC) {
    float m[JC], l[JC];
    float4 o[JC][DC];
#pragma unroll
    for (int c = 0; c < JC; ++c) {
      const int j = j0 + c;
      l[c] = j < p.nq ? red_l[j] + red_l[NQP + j] + red_l[2 * NQP + j] + red_l[3 * NQP + j] : 0.f;
      m[c] = l[c] > 0.f ? stash_m[j] : -INFINITY;
#pragma unroll
      for (int k = 0; k < DC; ++k)
        o[c][k] = l[c] > 0.f ? *reinterpret_cast<const float4*>(stash + j * DIM + k * D + 4 * lane)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll 1
    for (int s = 0; s < nseg; ++s) {
      if (s == own) continue;
      float2 e[JC];
      float4 v[JC][DC];
#pragma unroll
      for (int c = 0; c < JC; ++c) {
        const int j = j0 + c;
        if (j < p.nq) {
          const int64_t part = part_index(p, g, j, h, s, seg0);
          e[c] = __ldcg(ml + part);
#pragma unroll
          for (int k = 0; k < DC; ++k)
            v[c][k] = __ldcg(reinterpret_cast<const float4*>(p.part_o + part * DIM + k * D) + lane);
        } else {
          e[c] = make_float2(0.f, 0.f);
#pragma unroll
          for (int k = 0; k < DC; ++k) v[c][k] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
#pragma unroll
      for (int c = 0; c < JC; ++c) {
        if (e[c].y > 0.f) {
          const float mn = fmaxf(m[c], e[c].x);
          const float a = ex2(m[c] - mn), b = ex2(e[c].x - mn);
#pragma unroll
          for (int k = 0; k < DC; ++k)
            o[c][k] = make_float4(fmaf(o[c][k].x, a, v[c][k].x * b), fmaf(o[c][k].y, a, v[c][k].y * b),
                                  fmaf(o[c][k].z, a, v[c][k].z * b), fmaf(o[c][k].w, a, v[c][k].w * b));
          l[c] = fmaf(l[c], a, e[c].y * b);
          m[c] = mn;
        }
      }
    }
#pragma unroll
    for (int c = 0; c < JC; ++c) {
      const int j = j0 + c;
      if (j < p.nq) {
        const int64_t rowh = ((int64_t)g * p.nq + j) * p.heads + h;
#pragma unroll
        for (int k = 0; k < DC; ++k)
          store_out4(p.out + rowh * DIM + k * D + 4 * lane, o[c][k], l[c] > 0.f ? 1.f / l[c] : 0.f);
      }
    }
  }
}

// Running merge of segments for JC query columns (lane l holds dims 4l .. 4l+3 of each 128-dim chunk): max (log2
// units), sum, output. The merge is the combine's: out = sum_s w_s o_s / sum_s w_s l_s, w_s = 2^(m_s - max); a segment
// that saw no key (sum 0) takes no part, whatever its max.
template <int JC, int DC>
struct SegAcc {
  float m[JC], l[JC];
  float4 o[JC][DC];
  OMNI_DEV void clear() {
#pragma unroll
    for (int c = 0; c < JC; ++c) {
      m[c] = -INFINITY;
      l[c] = 0.f;
#pragma unroll
      for (int k = 0; k < DC; ++k) o[c][k] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  }
  OMNI_DEV void add(int c, float em, float el, const float4* ev) {
    if (el > 0.f) {
      const float mn = fmaxf(m[c], em);
      const float a = ex2(m[c] - mn), b = ex2(em - mn);
#pragma unroll
      for (int k = 0; k < DC; ++k)
        o[c][k] = make_float4(fmaf(o[c][k].x, a, ev[k].x * b), fmaf(o[c][k].y, a, ev[k].y * b),
                              fmaf(o[c][k].z, a, ev[k].z * b), fmaf(o[c][k].w, a, ev[k].w * b));
      l[c] = fmaf(l[c], a, el * b);
      m[c] = mn;
    }
  }
};

// Adds the segments of unit (g, h), queries j0 .. j0+JC-1, other than `own`, from the partial arrays (read through
// L2: other CTAs wrote them). Segments go outermost so that the chunk's loads of one segment are all in flight.
template <int JC, int DIM>
OMNI_DEV void add_other_segments(SegAcc<JC, DIM / D>& acc, const Params& p, int g, int h, int j0, int own, int nseg,
                                 int64_t seg0, int lane) {
  constexpr int DC = DIM / D;
  const float2* ml = reinterpret_cast<const float2*>(p.part_ml);
#pragma unroll 1
  for (int s = 0; s < nseg; ++s) {
    if (s == own) continue;
    float2 e[JC];
    float4 v[JC][DC];
#pragma unroll
    for (int c = 0; c < JC; ++c) {
      const int j = j0 + c;
      if (j < p.nq) {
        const int64_t part = part_index(p, g, j, h, s, seg0);
        e[c] = __ldcg(ml + part);
#pragma unroll
        for (int k = 0; k < DC; ++k) v[c][k] = __ldcg(reinterpret_cast<const float4*>(p.part_o + part * DIM + k * D) + lane);
      } else {
        e[c] = make_float2(0.f, 0.f);
#pragma unroll
        for (int k = 0; k < DC; ++k) v[c][k] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int c = 0; c < JC; ++c) acc.add(c, e[c].x, e[c].y, v[c]);
  }
}

// Adds this CTA's own segment (its stash) and writes the unit's output rows j0 .. j0+JC-1.
template <int JC, int DIM>
OMNI_DEV void finish_unit(SegAcc<JC, DIM / D>& acc, const Params& p, int g, int h, int j0, int lane, const float* red_l,
                          const float* stash_m, const float* stash) {
  constexpr int DC = DIM / D;
#pragma unroll
  for (int c = 0; c < JC; ++c) {
    const int j = j0 + c;
    if (j < p.nq) {
      const float l = red_l[j] + red_l[NQP + j] + red_l[2 * NQP + j] + red_l[3 * NQP + j];
      float4 own[DC];
#pragma unroll
      for (int k = 0; k < DC; ++k) own[k] = *reinterpret_cast<const float4*>(stash + j * DIM + k * D + 4 * lane);
      acc.add(c, stash_m[j], l, own);
      const int64_t rowh = ((int64_t)g * p.nq + j) * p.heads + h;
#pragma unroll
      for (int k = 0; k < DC; ++k)
        store_out4(p.out + rowh * DIM + k * D + 4 * lane, acc.o[c][k], acc.l[c] > 0.f ? 1.f / acc.l[c] : 0.f);
    }
  }
}

// S^T[buf] (+)= K chunk (slot) . Q chunk^T (thread 0): the keys' 128-dim chunk `chunk` of the head; chunks after the
// first accumulate.
OMNI_DEV void issue_scores(uint32_t tbase, int buf, const unsigned char* kslot, const unsigned char* qs, int chunk) {
  const uint32_t kaddr = smem_addr(kslot);
  const uint32_t qaddr = smem_addr(qs);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint64_t a = smem_desc(kaddr + (kk >> 2) * BOX_BYTES + (kk & 3) * 32, 16, 1024, kLayoutSw128);
    const uint64_t b =
        smem_desc(qaddr + (2 * chunk + (kk >> 2)) * (NQP * 128) + (kk & 3) * 32, 16, 1024, kLayoutSw128);
    mma_bf16_ss(tbase + buf * NQP, a, b, IDESC_S, (chunk > 0 || kk > 0) ? 1u : 0u);
  }
}

// O^T chunk (TMEM column dcol) = V chunk^T (slot) . P^T[buf]  (thread 0).
OMNI_DEV void issue_values(uint32_t tbase, uint32_t dcol, const unsigned char* vslot, const unsigned char* pbuf) {
  const uint32_t vaddr = smem_addr(vslot);
  const uint32_t paddr = smem_addr(pbuf);
#pragma unroll
  for (int kk = 0; kk < BN / 16; ++kk) {
    const uint64_t a = smem_desc(vaddr + kk * 2048, BOX_BYTES, 1024, kLayoutSw128);
    const uint64_t b = smem_desc(paddr + kk * 256, 128, 2048, kLayoutNone);
    mma_bf16_ss(tbase + dcol, a, b, IDESC_O, kk > 0 ? 1u : 0u);
  }
}

// NQT: query columns processed (a compile-time bound >= nq; the MMA always computes 16). SLOTS: ring slots (K and V of
// SLOTS / 2 tiles in flight; six fill the shared memory of one CTA per SM).
//
// Roles and their handshakes (mbarriers; b = tile & 1, u = tile >> 1 its use of buffer b):
//   producer (warp 4)   full[slot]  <- TMA bytes           empty[slot] -> refill
//   MMA (warp 5)        s_full[b]   <- S^T(tile) done      o_full[b]   <- O^T(tile) done
//   softmax (warps 0-3) s_free[b], p_full[b], o_free[b] (128 arrivals each)
//   queries (TMA by the producer, two buffers by unit parity): q_fill[q] <- bytes, q_done[q] <- unit's last S^T
// DIM: head_dim, 128 or 512. A key tile is DIM / 128 chunks of 128 dims, each a ring slot of 32 KB: S^T accumulates
// over the K chunks, O^T has one accumulator per V chunk. With more than one chunk, warp 8 zeroes the V rows past a
// unit's keys in each chunk of its last tile (vfix[c] <- zeroed) before the MMA reads them.
template <int NQT, int SLOTS, int DIM>
__global__ void __launch_bounds__(threads_for(DIM, NQT), 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap_half,
                   const __grid_constant__ CUtensorMap vmap_half, const Params pin) {
  using L = Smem<SLOTS, DIM>;
  constexpr int DC = DIM / D;  // 128-dim chunks per head
  constexpr int THREADS = threads_for(DIM, NQT);
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[SLOTS], empty[SLOTS];
  __shared__ __align__(8) uint64_t s_full[2], s_free[2], p_full[2], o_full[2], o_free[2], q_fill[2], q_done[2], drain;
  __shared__ __align__(8) uint64_t seg_ready, seg_free;  // the stash holds a finished unit / was written out
  __shared__ __align__(8) uint64_t vfix[DC];   // head_dim 512: a last tile's V chunk c has its stale rows zeroed
  __shared__ __align__(8) uint64_t vtail[DC];  // ... and its load was issued (so its slot's phase is the current one)
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ volatile int issued_k, issued_v, q_issued;  // K / V tiles and query tiles the producers issued

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  // Set-up that reads nothing an earlier kernel writes: barriers, TMEM, the tensor maps. Launched as a
  // programmatic dependent, this overlaps the previous kernel's tail.
  if (tid == 0) {
    OMNI_TRACE_AT(4002);
    for (int s = 0; s < SLOTS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&o_full[s], 1);
      mbar_init(&s_free[s], 128);
      mbar_init(&p_full[s], 128);
      mbar_init(&o_free[s], 128);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&q_fill[s], 1);
      mbar_init(&q_done[s], 1);
    }
    mbar_init(&drain, split_issue(DIM, NQT) ? 2 : 1);
    mbar_init(&seg_ready, 128);
    mbar_init(&seg_free, 1);
    for (int c = 0; c < DC; ++c) {
      mbar_init(&vfix[c], 1);
      mbar_init(&vtail[c], 1);
    }
    mbar_fence_init();
    abort_flag = 0;
    issued_k = issued_v = q_issued = 0;
  }
  if (warp == 0) tmem_alloc(&tmem_base, tmem_cols(DIM));
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&kmap);
    prefetch_tmap(&qmap);
  }
  if (warp == 6 && lane == 0) prefetch_tmap(&vmap);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (tid == 0) OMNI_TRACE_AT(4000);
  // The queries, the cache rows and the lengths may come from the kernel before this one.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // The lengths, read by every role's walk, once into shared memory, with the groups' cost prefix (thread g
  // computes group g's cost; a block-wide scan sums them).
  static_assert(kSmemGroups <= THREADS, "one thread per group for the cost prefix");
  __shared__ int64_t s_len[kSmemGroups];
  __shared__ int64_t s_pre[kSmemGroups + 1];
  __shared__ int64_t s_wsum[THREADS / 32];
  Params p = pin;
  const int64_t* pre_tab = nullptr;
  if (p.groups <= kSmemGroups) {
    int64_t c = 0;
    if (tid < p.groups) {
      const int64_t len = group_len(pin, tid);
      s_len[tid] = len;
      int64_t n = len + (p.causal ? p.nq - 1 : 0);
      n = n < 0 ? 0 : (n > p.cap ? p.cap : n);
      c = unit_cost(p, (n + BN - 1) / BN) * p.heads;
    }
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int64_t y = __shfl_up_sync(0xffffffffu, c, off);
      if (lane >= off) c += y;
    }
    if (lane == 31) s_wsum[warp] = c;
    __syncthreads();
    for (int w = 0; w < warp; ++w) c += s_wsum[w];
    if (tid < p.groups) s_pre[tid + 1] = c;
    if (tid == 0) s_pre[0] = 0;
    __syncthreads();
    p.lengths = s_len;
    pre_tab = s_pre;
  }
  if (tid == 0) OMNI_TRACE_AT(4003);
  const bool merge_here = p.counters != nullptr && p.out != nullptr;  // no combine kernel follows
  if (merge_here) {
    // What the combine would otherwise do for the units without a segment: report lengths outside the cache and
    // give the rows that see no key zeros (their units have no tiles, so no CTA of the pass visits them).
    if (blockIdx.x == 0) {
      for (int g = tid; g < p.groups && !p.prefill; g += THREADS) {  // prefill mode clamps its padding rows
        const int64_t raw = p.lengths[g] + (p.causal ? p.nq - 1 : 0);
        if (p.lengths[g] < 0 || raw > p.cap) raise_status(p.status, kStatusIndex);
      }
    }
    if (warp == 7) {
      for (int g = blockIdx.x; g < p.groups; g += gridDim.x) {
        if (unit_need(p, g) > 0) continue;
        uint4* o = reinterpret_cast<uint4*>(p.out + (int64_t)g * p.nq * p.heads * D);
        for (int i = lane; i < p.nq * p.heads * (D / 8); i += 32) o[i] = make_uint4(0u, 0u, 0u, 0u);
      }
    }
  }

  const int64_t total = pre_tab ? pre_tab[p.groups] : total_cost(p);
  if (tid == 0) OMNI_TRACE_AT(4007);
  // At least one tile's cost per CTA, so that every CTA between a unit's first and last owns one of its tiles.
  const int64_t per = max((total + gridDim.x - 1) / gridDim.x, kTileCost);
  const int64_t c0 = (int64_t)blockIdx.x * per;
  const int64_t c1 = min(total, c0 + per);
  TileIter first_tile;  // this CTA's first tile; every role starts its walk from a copy
  first_tile.init(p, c0, c1, pre_tab);
  const bool has_work = c0 < c1 && !first_tile.done;  // uniform over the CTA
  if (tid == 0) OMNI_TRACE_AT(4008);
  OMNI_TRACE_CTA(0);
  if (tid == 0) {
    OMNI_TRACE_AT(4001);
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the combine may start its prologue
  }
  const uint32_t tbase = tmem_base;
  unsigned char* qs = smem + L::Q_OFF;

  constexpr int HALF = SLOTS / 2;
  if (!has_work) {
    // nothing to do but give the TMEM back
  } else if (warp == 4 || warp == 6) {
    // ------------------------------------------------------------------ producers: K (+ queries) and V
    if (lane == 0) {
      const bool is_k = warp == 4;
      const CUtensorMap* map = is_k ? &kmap : &vmap;
      const CUtensorMap* map_half = is_k ? &kmap_half : &vmap_half;  // 64-row boxes, for short unit tails
      prefetch_tmap(map_half);
      TileIter ti = first_tile, ahead = first_tile;  // `ahead` runs p.prefetch tiles in front (into L2 early)
      for (int i = 0; i < p.prefetch && !ahead.done; ++i) ahead.advance();
      if (is_k) OMNI_TRACE_AT(4005);
      int unit = 0;
      for (int it = 0; !ti.done && !abort_flag; ++it, ti.advance()) {
        const int h = ti.h, tt = ti.t;
        if (p.prefetch > 0 && !ahead.done) {
          tma_prefetch_4d(map, 0, ahead.t * BN, ahead.h, ahead.g);
          tma_prefetch_4d(map, 64, ahead.t * BN, ahead.h, ahead.g);
          ahead.advance();
        }
        if (is_k && (tt == 0 || it == 0)) {
          // The unit's queries (16 rows of head h from row g * nq; rows past the group are masked later).
          const int qb = unit & 1;
          if (unit >= 2 && !mbar_wait(&q_done[qb], ((unit >> 1) - 1) & 1)) {
            abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&q_fill[qb], NQP * DIM * 2);
#pragma unroll
          for (int bx = 0; bx < DIM / 64; ++bx)
            tma_load_3d(qs + qb * (NQP * DIM * 2) + bx * (NQP * 128), &qmap, bx * 64, h, ti.g * p.nq, &q_fill[qb]);
          q_issued = ++unit;
          if (unit == 1) OMNI_TRACE_AT(4006);
        }
        // A unit's last tile with at most 64 keys left loads 64-row boxes: the rows past the keys are masked (K) or
        // zeroed (V: by the softmax warps for head_dim 128, by warp 8 otherwise) whatever they hold.
        const bool short_tail = (int64_t)tt * BN + 64 >= ti.need;
        const CUtensorMap* m = short_tail ? map_half : map;
        bool stop = false;
#pragma unroll 1
        for (int c = 0; c < DC; ++c) {  // the tile's 128-dim chunks, one ring slot each
          const int ci = it * DC + c;
          const int slot = (is_k ? 0 : HALF) + ci % HALF, use = ci / HALF;
          if (use >= 1 && !mbar_wait(&empty[slot], (use - 1) & 1)) {
            abort_flag = 1;
            stop = true;
            break;
          }
          mbar_arrive_expect_tx(&full[slot], short_tail ? SLOT_BYTES / 2 : SLOT_BYTES);
          const int crow = ti.g / p.kv_div;  // the group's cache row
          tma_load_4d(smem + slot * SLOT_BYTES, m, c * D, tt * BN, h, crow, &full[slot]);
          tma_load_4d(smem + slot * SLOT_BYTES + BOX_BYTES, m, c * D + 64, tt * BN, h, crow, &full[slot]);
          if (is_k) {
            issued_k = ci + 1;
          } else {
            issued_v = ci + 1;
            // A last tile's V chunk: warp 8 may now wait for its load (the slot's current phase is this chunk's).
            if (DC > 1 && (int64_t)tt * BN + BN > ti.need) mbar_arrive(&vtail[c]);
          }
        }
        if (stop) break;
        if (is_k) OMNI_TRACE_AT(it * 8);
        else OMNI_TRACE_AT(it * 8 + 1);
      }
    }
    __syncwarp();
  } else if (warp == 5 || (split_issue(DIM, NQT) && warp == pv_warp(DIM))) {
    // ------------------------------------------------------------------ MMA issuer(s)
    if (lane == 0 && warp == pv_warp(DIM)) {
      // ---------------------------------------------------------------- O^T issuer (split issue)
      TileIter ti = first_tile;
      int unit = -1;
      (void)unit;
      // O^T(t) = V(t)^T P^T(t), one accumulator per 128-dim chunk. tail: the index of this tile among the CTA's last
      // tiles of units (head_dim 512: its V chunks wait until warp 8 has zeroed their stale rows), or -1.
      auto values = [&](int t, int tail) -> bool {
        const int b = t & 1, u = t >> 1;
        if (u >= 1 && !mbar_wait(&o_free[b], (u - 1) & 1)) return false;
        if (!mbar_wait(&p_full[b], u & 1)) return false;
#pragma unroll 1
        for (int c = 0; c < DC; ++c) {
          const int ci = t * DC + c;
          const int slot = HALF + ci % HALF;
          if (DC > 1 && tail >= 0) {
            if (!mbar_wait(&vfix[c], tail & 1)) return false;
          } else if (!mbar_wait(&full[slot], (ci / HALF) & 1)) {
            return false;
          }
          tc_fence_after();
          if (c == 0) OMNI_TRACE_AT(t * 8 + 3);
          issue_values(tbase, ocol(b, c, DC), smem + slot * SLOT_BYTES, smem + L::P_OFF + b * (NQP * BN * 2));
          if (c == DC - 1) tc_commit(&o_full[b]);
          tc_commit(&empty[slot]);
        }
        return true;
      };
      bool ok = true;
      int tails = 0;
      for (int it = 0; !ti.done && ok && !abort_flag; ++it, ti.advance()) {
        const int tail = DC > 1 && (int64_t)ti.t * BN + BN > ti.need ? tails++ : -1;
        ok = values(it, tail);
      }
      if (!ok) abort_flag = 1;
    } else if (lane == 0) {
      TileIter ti = first_tile;
      int unit = -1;
      auto scores = [&](int t) -> bool {  // S^T(t) = K(t) Q^T, accumulated over the head's 128-dim chunks
        const int b = t & 1, u = t >> 1;
        if (u >= 1 && !mbar_wait(&s_free[b], (u - 1) & 1)) return false;
#pragma unroll 1
        for (int c = 0; c < DC; ++c) {
          const int ci = t * DC + c;
          const int slot = ci % HALF;
          if (!mbar_wait(&full[slot], (ci / HALF) & 1)) return false;
          tc_fence_after();
          if (c == 0) OMNI_TRACE_AT(t * 8 + 2);
          issue_scores(tbase, b, smem + slot * SLOT_BYTES, qs + (unit & 1) * (NQP * DIM * 2), c);
          if (c == DC - 1) tc_commit(&s_full[b]);
          tc_commit(&empty[slot]);
        }
        return true;
      };
      // O^T(t) = V(t)^T P^T(t), one accumulator per 128-dim chunk. tail: the index of this tile among the CTA's last
      // tiles of units (head_dim 512: its V chunks wait until warp 8 has zeroed their stale rows), or -1.
      auto values = [&](int t, int tail) -> bool {
        const int b = t & 1, u = t >> 1;
        if (u >= 1 && !mbar_wait(&o_free[b], (u - 1) & 1)) return false;
        if (!mbar_wait(&p_full[b], u & 1)) return false;
#pragma unroll 1
        for (int c = 0; c < DC; ++c) {
          const int ci = t * DC + c;
          const int slot = HALF + ci % HALF;
          if (DC > 1 && tail >= 0) {
            if (!mbar_wait(&vfix[c], tail & 1)) return false;
          } else if (!mbar_wait(&full[slot], (ci / HALF) & 1)) {
            return false;
          }
          tc_fence_after();
          if (c == 0) OMNI_TRACE_AT(t * 8 + 3);
          issue_values(tbase, ocol(b, c, DC), smem + slot * SLOT_BYTES, smem + L::P_OFF + b * (NQP * BN * 2));
          if (c == DC - 1) tc_commit(&o_full[b]);
          tc_commit(&empty[slot]);
        }
        return true;
      };
      bool ok = true;
      if constexpr (split_issue(DIM, NQT)) {
        // S^T only: the O^T issuer (warp pv_warp) walks the same tiles on its own.
        for (int it = 0; !ti.done && ok && !abort_flag; ++it, ti.advance()) {
          if (ti.t == 0 || it == 0) {
            ++unit;
            if (!mbar_wait(&q_fill[unit & 1], (unit >> 1) & 1)) ok = false;
          }
          if (ok) ok = scores(it);
          if (ok && ti.last_here()) tc_commit(&q_done[unit & 1]);  // the unit's last S^T in this CTA
        }
      } else {
        // Tile t's S^T goes out before tile t-1's O^T, so the softmax of t can start while O^T(t-1) runs -- also
        // across a unit boundary, where the softmax finishes the old unit one tile late.
        int pend = -1;       // tile whose O^T is still to issue
        int pend_tail = -1;  // its index among the last tiles of units (head_dim 512), or -1
        int tails = 0;
        for (int it = 0; !ti.done && ok && !abort_flag; ++it, ti.advance()) {
          if (ti.t == 0 || it == 0) {
            ++unit;
            if (!mbar_wait(&q_fill[unit & 1], (unit >> 1) & 1)) ok = false;
          }
          if (ok) ok = scores(it);
          if (ok && ti.last_here()) tc_commit(&q_done[unit & 1]);  // the unit's last S^T in this CTA
          if (ok && pend >= 0) ok = values(pend, pend_tail);
          pend = it;
          pend_tail = DC > 1 && (int64_t)ti.t * BN + BN > ti.need ? tails++ : -1;
        }
        if (ok && pend >= 0 && !abort_flag) ok = values(pend, pend_tail);
      }
      if (!ok) abort_flag = 1;
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------------------------ softmax (128 threads, TMEM lane = tid)
    // The running max of a column is raised only when a score passes it by 2^8, so the cross-thread max (and the
    // rescale of the accumulators) is rare; O^T of a tile is accumulated one tile later.
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    float* red = reinterpret_cast<float*>(smem + L::RED_OFF);
    TileIter ti = first_tile;
    float* red_l = reinterpret_cast<float*>(smem + L::RED_L_OFF);
    float* stash_m = reinterpret_cast<float*>(smem + L::STASH_M_OFF);
    float* stash = reinterpret_cast<float*>(smem + L::STASH_OFF);
    float m[NQT], lpart[NQT], acc[DC][NQT], scl[NQT];  // acc: thread = head dim (c * 128 + tid) of chunk c
    int lim[NQT];
    int g = 0, h = 0, need = 0, tiles = 1;
    int64_t unit_pos0 = 0;
    bool pending = false;
    bool stashed = false;  // a finished unit waits for its last O^T (read at the next tile)
    int segs = 0;          // finished units handed to the write-out warp
    for (int it = 0; !ti.done; ++it, ti.advance()) {
      const int tt = ti.t;
      const int b = it & 1;
      const uint32_t par = (it >> 1) & 1;
      const bool first = tt == 0 || it == 0;
      const bool last = ti.last_here();
      if (first) {
        g = ti.g;
        h = ti.h;
        tiles = (int)ti.tiles;
        need = (int)ti.need;
        unit_pos0 = ti.unit_pos0();
        const int64_t n = group_len(p, g);
#pragma unroll
        for (int j = 0; j < NQT; ++j) {
          int64_t lj = n + (p.causal ? j : 0);
          lj = lj < 0 ? 0 : lj;
          lim[j] = j < p.nq ? (int)(lj > need ? need : lj) : 0;
          m[j] = 0.f;  // a guess; the first tile lowers it if its scores are far below, or raises it
          lpart[j] = 0.f;
#pragma unroll
          for (int c = 0; c < DC; ++c) acc[c][j] = 0.f;
        }
      }
      const int key = tt * BN + tid;
      if (tid == 0) OMNI_TRACE_AT(it * 8 + 7);

      // Scores of this tile.
      if (!mbar_wait(&s_full[b], par)) abort_flag = 1;
      if (tid == 0) OMNI_TRACE_AT(it * 8 + 4);
      tc_fence_after();
      __syncwarp();
      float s[NQP];
      tmem_ld16(tbase + lane_off + b * NQP, s);
      tc_fence_before();
      mbar_arrive(&s_free[b]);
      float xv[NQT];
      bool over = false;
#pragma unroll
      for (int j = 0; j < NQT; ++j) {
        xv[j] = key < lim[j] ? s[j] * p.qscale : -INFINITY;
        over |= xv[j] > m[j] + kRescale;
        if (first) over |= xv[j] > -INFINITY && xv[j] < m[j] - kBelow;
      }
      // One barrier per tile: does any thread need a new max, or has any seen an abort? (Both take the slow
      // path, whose barrier then decides the abort from the values each thread read before the first one.)
      const bool saw_abort = abort_flag != 0;
      if (named_sync_or(1, 128, over || saw_abort)) {
        {
          int col;
          const float v = butterfly<NQT, true>(xv, lane, col);
          if (butterfly_writer<NQT>(lane)) red[warp * NQP + col] = v;
        }
        if (named_sync_or(1, 128, saw_abort)) break;
#pragma unroll
        for (int j = 0; j < NQT; ++j) {
          const float tmax = fmaxf(fmaxf(red[j], red[NQP + j]), fmaxf(red[2 * NQP + j], red[3 * NQP + j]));
          // First tile of the unit here: nothing is accumulated yet, so the max may also go down.
          const float mnew = first ? (tmax == -INFINITY ? m[j] : tmax) : fmaxf(m[j], tmax);
          scl[j] = ex2(m[j] - mnew);
          m[j] = mnew;
#pragma unroll
          for (int c = 0; c < DC; ++c) acc[c][j] *= scl[j];
          lpart[j] *= scl[j];
        }
        named_sync(1, 128);
      } else {
#pragma unroll
        for (int j = 0; j < NQT; ++j) scl[j] = 1.f;
      }
      float pr[NQP];
#pragma unroll
      for (int j = 0; j < NQP; ++j) pr[j] = 0.f;
#pragma unroll
      for (int j = 0; j < NQT; ++j) {
        pr[j] = ex2(xv[j] - m[j]);
        lpart[j] += pr[j];
      }
      {
        unsigned char* pb = smem + L::P_OFF + b * (NQP * BN * 2);
        uint32_t wv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(pr[2 * i]));
          const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(pr[2 * i + 1]));
          wv[i] = lo | (hi << 16);
        }
        *reinterpret_cast<uint4*>(pb + tid * 16) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        *reinterpret_cast<uint4*>(pb + 2048 + tid * 16) =
            NQT > 8 ? make_uint4(wv[4], wv[5], wv[6], wv[7]) : make_uint4(0u, 0u, 0u, 0u);
      }
      // A tile that ends inside the unit's keys: zero the V rows past them (they may hold anything). With more than
      // one chunk per tile, warp 8 does this.
      if (DC == 1 && tt * BN + BN > need) {
        const int vslot = HALF + it % HALF;
        if (!mbar_wait(&full[vslot], (it / HALF) & 1)) abort_flag = 1;
        if (key >= need) {
          unsigned char* row = smem + vslot * SLOT_BYTES + tid * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            *reinterpret_cast<uint4*>(row + c * 16) = make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(row + BOX_BYTES + c * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
        }
      }
      fence_async_smem();
      mbar_arrive(&p_full[b]);
      if (tid == 0) OMNI_TRACE_AT(it * 8 + 5);

      // The previous tile's O^T: brought to this tile's max -- or, when the previous tile ended a unit, added to
      // that unit's stashed accumulator, which then becomes the unit's segment (or output).
      if (pending) {
        if (!mbar_wait(&o_full[b ^ 1], ((it - 1) >> 1) & 1)) abort_flag = 1;
        if (tid == 0) OMNI_TRACE_AT(it * 8 + 6);
        tc_fence_after();
        __syncwarp();
        float o[DC][NQP];
#pragma unroll
        for (int c = 0; c < DC; ++c) tmem_ld16(tbase + lane_off + ocol(b ^ 1, c, DC), o[c]);
        tc_fence_before();
        mbar_arrive(&o_free[b ^ 1]);
        if (stashed) {
#pragma unroll
          for (int c = 0; c < DC; ++c)
#pragma unroll
            for (int j = 0; j < NQT; ++j) stash[j * DIM + c * D + tid] += o[c][j];
          mbar_arrive(&seg_ready);  // the write-out warp takes it from here
          ++segs;
          stashed = false;
        } else {
#pragma unroll
          for (int c = 0; c < DC; ++c)
#pragma unroll
            for (int j = 0; j < NQT; ++j) acc[c][j] = fmaf(scl[j], o[c][j], acc[c][j]);
        }
      }
      pending = true;

      if (last) {
        // End of this CTA's part of the unit: its column sums, maximum and accumulator go to the stash once the
        // write-out warp is done with the previous unit; its last O^T is added one tile later when this CTA has
        // more tiles (at once otherwise), and the write-out warp turns the stash into the segment (or output).
        if (segs >= 1 && !mbar_wait_or(&seg_free, (segs - 1) & 1, &abort_flag)) abort_flag = 1;
        {
          int col;
          const float v = butterfly<NQT, false>(lpart, lane, col);
          if (butterfly_writer<NQT>(lane)) red_l[warp * NQP + col] = v;
        }
        if (tid == 0) {
#pragma unroll
          for (int j = 0; j < NQT; ++j) stash_m[j] = m[j];  // the same in every thread
        }
        TileIter nx = ti;
        nx.advance();
        if (!nx.done) {
#pragma unroll
          for (int c = 0; c < DC; ++c)
#pragma unroll
            for (int j = 0; j < NQT; ++j) stash[j * DIM + c * D + tid] = acc[c][j];
          stashed = true;
        } else {
          if (!mbar_wait(&o_full[b], par)) abort_flag = 1;
          tc_fence_after();
          __syncwarp();
          float o[DC][NQP];
#pragma unroll
          for (int c = 0; c < DC; ++c) tmem_ld16(tbase + lane_off + ocol(b, c, DC), o[c]);
          tc_fence_before();
          mbar_arrive(&o_free[b]);
#pragma unroll
          for (int c = 0; c < DC; ++c)
#pragma unroll
            for (int j = 0; j < NQT; ++j) stash[j * DIM + c * D + tid] = acc[c][j] + o[c][j];
          pending = false;
          mbar_arrive(&seg_ready);
          ++segs;
        }
        if (tid == 0) OMNI_TRACE_AT(4010 + (it & 7));
      }
    }
  } else if (warp == 7) {
    // ------------------------------------------------------------------ write-out of finished units
    // Walks this CTA's tiles like the other roles; at a unit's last tile here, waits for the softmax warps'
    // stash and writes the unit's segment (or output row): lane l holds dimensions 4l .. 4l+3.
    const float* red_l = reinterpret_cast<const float*>(smem + L::RED_L_OFF);
    const float* stash_m = reinterpret_cast<const float*>(smem + L::STASH_M_OFF);
    const float* stash = reinterpret_cast<const float*>(smem + L::STASH_OFF);
    if constexpr (NQT <= 2) {
      // Decode (one or two queries per unit): while it waits for the stash, this warp watches the unit's counter
      // (every lane loads it with acquire semantics, one L2 request); once every other CTA of the unit has
      // counted, this CTA is the unit's last, and the others' segments are merged in registers before the stash
      // is ready, so that only its own segment and the stores remain (measured: 3 % off the decode step). With
      // more queries the same code slowed the softmax warps' steady state (the kernel's register allocation
      // changes), so those keep the plain path below.
      constexpr int JC = NQT;
      int segs = 0;
      for (TileIter ti = first_tile; !ti.done; ti.advance()) {
        if (!ti.last_here()) continue;
        const int64_t pos0 = ti.unit_pos0();
        const int64_t seg0 = pos0 / per;  // the unit's first CTA
        const int seg = (int)(blockIdx.x - seg0);
        const int nseg = (int)((pos0 + kTileCost * (ti.tiles - 1)) / per - seg0 + 1);
        const bool whole = nseg == 1;
        unsigned* ctr = merge_here && !whole ? p.counters + (int64_t)ti.g * p.heads + ti.h : nullptr;
        SegAcc<JC, DC> acc;
        acc.clear();
        bool last = false;  // this CTA merges the unit
        // Only the unit's first CTA watches: it works on the unit at the end of its range, the others at the start of
        // theirs, so it is normally the last. The polls are spaced out (the spinning warp shares its SM sub-partition
        // with a softmax warp); decisions are taken from lane 0's view, so that the warp stays converged.
        if (ctr && seg == 0) {
          const uint64_t t0 = global_ns();
          while (!__shfl_sync(0xffffffffu, mbar_test_wait(&seg_ready, segs & 1), 0)) {
            if (__shfl_sync(0xffffffffu, abort_flag != 0 || global_ns() - t0 > kWaitLimitNs, 0)) break;
            if (__shfl_sync(0xffffffffu, ld_acquire_gpu(ctr), 0) == (unsigned)(nseg - 1)) {
              add_other_segments<JC, DIM>(acc, p, ti.g, ti.h, 0, seg, nseg, seg0, lane);
              last = true;
              break;
            }
            __nanosleep(256);
          }
        }
        if (!mbar_wait_or(&seg_ready, segs & 1, &abort_flag)) {
          abort_flag = 1;
          break;
        }
        bool counted = false;  // last, found after the stash was ready: the others' segments are still to be read
        if (ctr && !last) counted = last = __shfl_sync(0xffffffffu, ld_acquire_gpu(ctr), 0) == (unsigned)(nseg - 1);
        if (!last) {
          for (int j = 0; j < p.nq && j < NQT; ++j) {
            const float l = red_l[j] + red_l[NQP + j] + red_l[2 * NQP + j] + red_l[3 * NQP + j];
            const int64_t rowh = ((int64_t)ti.g * p.nq + j) * p.heads + ti.h;
            const int64_t part = part_index(p, ti.g, j, ti.h, seg, seg0);
#pragma unroll
            for (int c = 0; c < DC; ++c) {
              const float4 a = *reinterpret_cast<const float4*>(stash + j * DIM + c * D + 4 * lane);
              if (whole && p.out) store_out4(p.out + rowh * DIM + c * D + 4 * lane, a, l > 0.f ? 1.f / l : 0.f);
              else *reinterpret_cast<float4*>(p.part_o + part * DIM + c * D + 4 * lane) = a;
            }
            if (!(whole && p.out) && lane == 0) reinterpret_cast<float2*>(p.part_ml)[part] = make_float2(stash_m[j], l);
          }
          if (ctr) {
            __threadfence();  // this lane's partial stores before the count
            __syncwarp();
            unsigned old = 0;
            if (lane == 0) old = atomicAdd(ctr, 1u);
            counted = last = __shfl_sync(0xffffffffu, old, 0) == (unsigned)(nseg - 1);
            if (last) __threadfence();  // the other CTAs' partials after their counts
          }
        }
        if (last) {
          if (counted) add_other_segments<JC, DIM>(acc, p, ti.g, ti.h, 0, seg, nseg, seg0, lane);  // else merged
          finish_unit<JC, DIM>(acc, p, ti.g, ti.h, 0, lane, red_l, stash_m, stash);
          if (lane == 0) *ctr = 0;  // zero again for the next call
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&seg_free);
        ++segs;
      }
    } else {
      int segs = 0;
      for (TileIter ti = first_tile; !ti.done; ti.advance()) {
        if (!ti.last_here()) continue;
        if (!mbar_wait_or(&seg_ready, segs & 1, &abort_flag)) {
          abort_flag = 1;
          break;
        }
        const int64_t pos0 = ti.unit_pos0();
        const int64_t seg0 = pos0 / per;  // the unit's first CTA
        const int seg = (int)(blockIdx.x - seg0);
        const int nseg = (int)((pos0 + kTileCost * (ti.tiles - 1)) / per - seg0 + 1);
        const bool whole = nseg == 1;
        // In-pass merge of a unit cut between CTAs: the segments are counted per unit; the CTA that finds the others
        // all published (one acquire load) merges at once from its stash without publishing its own, else it
        // publishes and counts, and the last to count merges.
        unsigned* ctr = merge_here && !whole ? p.counters + (int64_t)ti.g * p.heads + ti.h : nullptr;
        bool last = false;
        if (ctr) {
          unsigned c = 0;
          if (lane == 0) c = ld_acquire_gpu(ctr);
          last = __shfl_sync(0xffffffffu, c, 0) == (unsigned)(nseg - 1);
        }
        if (!last) {
          for (int j = 0; j < p.nq && j < NQT; ++j) {
            const float l = red_l[j] + red_l[NQP + j] + red_l[2 * NQP + j] + red_l[3 * NQP + j];
            const int64_t rowh = ((int64_t)ti.g * p.nq + j) * p.heads + ti.h;
            const int64_t part = part_index(p, ti.g, j, ti.h, seg, seg0);
#pragma unroll
            for (int c = 0; c < DC; ++c) {
              const float4 a = *reinterpret_cast<const float4*>(stash + j * DIM + c * D + 4 * lane);
              if (whole && p.out) store_out4(p.out + rowh * DIM + c * D + 4 * lane, a, l > 0.f ? 1.f / l : 0.f);
              else *reinterpret_cast<float4*>(p.part_o + part * DIM + c * D + 4 * lane) = a;
            }
            if (!(whole && p.out) && lane == 0) reinterpret_cast<float2*>(p.part_ml)[part] = make_float2(stash_m[j], l);
          }
          if (ctr) {
            __threadfence();  // this lane's partial stores before the count
            __syncwarp();
            unsigned old = 0;
            if (lane == 0) old = atomicAdd(ctr, 1u);
            last = __shfl_sync(0xffffffffu, old, 0) == (unsigned)(nseg - 1);
          }
        }
        if (last) {
          __threadfence();  // the other CTAs' partials after their counts
          merge_unit<NQT, DIM>(p, ti.g, ti.h, seg, nseg, seg0, lane, red_l, stash_m, stash);
          if (lane == 0) *ctr = 0;  // zero again for the next call
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&seg_free);
        ++segs;
      }
    }
  } else if (DC > 1 && warp == 8) {
    // ------------------------------------------------------------------ head_dim 512: stale V rows of last tiles
    // A unit's last tile may end inside the tile; the V rows past the unit's keys hold whatever the cache (or an
    // earlier load into the slot) holds there, possibly NaN, and P^T is zero there but 0 x NaN is NaN. For each V
    // chunk of such a tile: wait for its load, zero those rows (16-byte stores over the warp), make them visible to
    // the tensor core and hand the chunk to the MMA issuer (vfix[c]: one phase per such tile).
    // The chunk's load is awaited only after the V producer has issued it (vtail[c]): the warp walks its tiles
    // without waiting on the others, and a parity wait on a slot whose current phase is two behind would pass at once.
    int it = 0, tails = 0;
    for (TileIter ti = first_tile; !ti.done && !abort_flag; ti.advance(), ++it) {
      if ((int64_t)ti.t * BN + BN <= ti.need) continue;
      const int valid = (int)(ti.need - (int64_t)ti.t * BN);  // rows 0 .. valid-1 hold keys
      bool stop = false;
#pragma unroll 1
      for (int c = 0; c < DC; ++c) {
        const int ci = it * DC + c;
        const int slot = HALF + ci % HALF;
        if (!mbar_wait_or(&vtail[c], tails & 1, &abort_flag) || !mbar_wait_or(&full[slot], (ci / HALF) & 1, &abort_flag)) {
          abort_flag = 1;
          stop = true;
          break;
        }
        unsigned char* base = smem + slot * SLOT_BYTES;
        for (int i = lane; i < (BN - valid) * 16; i += 32) {  // 16 16-byte words per row: 8 in each 64-column box
          const int r = valid + (i >> 4), k = i & 15;
          *reinterpret_cast<uint4*>(base + (k >> 3) * BOX_BYTES + r * 128 + (k & 7) * 16) = make_uint4(0u, 0u, 0u, 0u);
        }
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&vfix[c]);
      }
      if (stop) break;
      ++tails;
    }
  }
  __syncthreads();
  if (tid == 0) OMNI_TRACE_AT(4020);
  if (abort_flag) {
    if (tid == 0) raise_status(p.status, kStatusTimeout);
    if (tid == 5 * 32 || (split_issue(DIM, NQT) && tid == pv_warp(DIM) * 32)) {
      tc_commit(&drain);  // every MMA the issuer thread(s) issued has completed once these arrive
      mbar_wait(&drain, 0);
    }
    if (tid == 4 * 32) {
      // Let the last load of every slot land before the CTA's shared memory goes away (a slot is refilled only
      // after its previous load completed and was consumed).
      for (int i = issued_k > HALF ? issued_k - HALF : 0; i < issued_k; ++i) mbar_wait(&full[i % HALF], (i / HALF) & 1);
      for (int i = issued_v > HALF ? issued_v - HALF : 0; i < issued_v; ++i)
        mbar_wait(&full[HALF + i % HALF], (i / HALF) & 1);
      for (int i = q_issued > 2 ? q_issued - 2 : 0; i < q_issued; ++i) mbar_wait(&q_fill[i & 1], (i >> 1) & 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, tmem_cols(DIM));
  }
  if (tid == 0) OMNI_TRACE_AT(4021);
  OMNI_TRACE_CTA(1);
}

// Merges the segments of each (query row, head): out = sum w_s o_s / sum w_s l_s. For beam search it first attends
// the row's generated keys itself (they do not depend on the pass, so this overlaps the pass's tail): warp w scores 8
// of each 32 keys (lane l holds dims 4l..4l+3 of every 128-dim chunk; all 8 loads in flight, then butterfly sums), and
// thread d accumulates dims d, d + 128, .. over the chunk's V rows; the result is one more segment. A unit the pass
// finished inside one CTA was written by the pass itself.
template <int DIM>
OMNI_DEV void combine_tc_body(const Params& p, int grid, __nv_bfloat16* __restrict__ out, const GenKeys& gen) {
  constexpr int DC = DIM / D;
  __shared__ long long red_total[4], red_pre[4];
  __shared__ long long unit_tiles;
  __shared__ float qs[DIM];
  __shared__ float sc[32];
  __shared__ long long koff[32];
  const int64_t rh = blockIdx.x;
  const int row = (int)(rh / p.heads);
  const int h = (int)(rh % p.heads);
  const int g = row / p.nq;
  const int t = threadIdx.x;
  const int warp = t >> 5, lane = t & 31;

  float gm = -INFINITY, gl = 0.f, go[DC];  // the generated keys' segment
#pragma unroll
  for (int c = 0; c < DC; ++c) go[c] = 0.f;
  if (gen.enabled) {
#pragma unroll
    for (int c = 0; c < DC; ++c) qs[c * D + t] = __bfloat162float(p.q[rh * DIM + c * D + t]);
    int64_t n = gen.gen_len[row];
    n = n < 0 ? 0 : (n > gen.cache_len ? gen.cache_len : n);
    __syncthreads();
    for (int64_t j0 = 0; j0 < n; j0 += 32) {
      uint2 kv[8][DC];
      long long off[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int64_t j = j0 + 8 * warp + i;
        int64_t src = row;
        if (j < n) {
          const int64_t pj = gen.ptr[(int64_t)row * gen.ptr_stride + j];
          if (pj < 0 || pj >= gen.cache_rows) {
            if (lane == 0) raise_status(p.status, kStatusIndex);
          } else {
            src = pj;
          }
        }
        off[i] = src * gen.s_kb + (int64_t)h * gen.s_kh + j * gen.s_ks;
#pragma unroll
        for (int c = 0; c < DC; ++c)
          kv[i][c] = j < n ? *reinterpret_cast<const uint2*>(gen.k + off[i] + c * D + 4 * lane) : make_uint2(0u, 0u);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float d = 0.f;
#pragma unroll
        for (int c = 0; c < DC; ++c) {
          const float* qc = qs + c * D + 4 * lane;
          d += __uint_as_float(kv[i][c].x << 16) * qc[0] + __uint_as_float(kv[i][c].x & 0xffff0000u) * qc[1] +
               __uint_as_float(kv[i][c].y << 16) * qc[2] + __uint_as_float(kv[i][c].y & 0xffff0000u) * qc[3];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
        if (lane == 0) {
          const int64_t j = j0 + 8 * warp + i;
          sc[8 * warp + i] = j < n ? d * p.qscale : -INFINITY;
          koff[8 * warp + i] = off[i];
        }
      }
      __syncthreads();
      float cm = -INFINITY;
#pragma unroll
      for (int i = 0; i < 32; ++i) cm = fmaxf(cm, sc[i]);
      const float mnew = fmaxf(gm, cm);
      const float scale = ex2(gm - mnew);  // 0 for the first chunk
#pragma unroll
      for (int c = 0; c < DC; ++c) go[c] *= scale;
      gl *= scale;
#pragma unroll
      for (int c = 0; c < DC; ++c) {
        __nv_bfloat16 vv[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) vv[i] = j0 + i < n ? gen.v[koff[i] + c * D + t] : __float2bfloat16_rn(0.f);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float pi = j0 + i < n ? ex2(sc[i] - mnew) : 0.f;
          if (c == 0) gl += pi;
          go[c] = fmaf(pi, __bfloat162float(vv[i]), go[c]);
        }
      }
      gm = mnew;
      __syncthreads();  // sc / koff are refilled by the next chunk
    }
  }

  long long tot = 0, pre = 0;
  for (int i = t; i < p.groups; i += 128) {
    const long long n = (unit_need(p, i) + BN - 1) / BN;
    const long long c = unit_cost(p, n) * p.heads;
    tot += c;
    if (i < g) pre += c;
    if (i == g) unit_tiles = n;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    tot += __shfl_xor_sync(0xffffffffu, tot, o);
    pre += __shfl_xor_sync(0xffffffffu, pre, o);
  }
  if ((t & 31) == 0) {
    red_total[t >> 5] = tot;
    red_pre[t >> 5] = pre;
  }
  __syncthreads();
  const long long total = red_total[0] + red_total[1] + red_total[2] + red_total[3];
  const long long tiles = unit_tiles;
  const long long pos0 =
      red_pre[0] + red_pre[1] + red_pre[2] + red_pre[3] + (long long)h * unit_cost(p, tiles) + p.unit_cost;
  if (t == 0 && h == 0 && row % p.nq == 0 && !p.prefill) {
    const int64_t raw = p.lengths[g] + (p.causal ? p.nq - 1 : 0);
    if (p.lengths[g] < 0 || raw > p.cap) raise_status(p.status, kStatusIndex);
  }
  const long long per = max((total + grid - 1) / grid, (long long)kTileCost);
  const int nseg = tiles > 0 ? (int)((pos0 + kTileCost * (tiles - 1)) / per - pos0 / per + 1) : 0;
  // The pass (and its partials) complete -- waited for by every block, so that the combine's completion implies
  // the pass's even when the pass finished every unit itself.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (nseg == 1 && !gen.enabled && p.out != nullptr) return;  // finished by the pass
  const float2* ml = reinterpret_cast<const float2*>(p.part_ml) + rh * p.st;
  // Segments that saw no key (sum 0) take no part, whatever their max.
  float mx = gl > 0.f ? gm : -INFINITY;
  for (int s = 0; s < nseg; ++s)
    if (ml[s].y > 0.f) mx = fmaxf(mx, ml[s].x);
  float o[DC], l = 0.f;
#pragma unroll
  for (int c = 0; c < DC; ++c) o[c] = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < nseg; ++s) {
      const float2 e = ml[s];
      if (e.y > 0.f) {
        const float wgt = ex2(e.x - mx);
#pragma unroll
        for (int c = 0; c < DC; ++c) o[c] = fmaf(wgt, p.part_o[(rh * p.st + s) * DIM + c * D + t], o[c]);
        l = fmaf(wgt, e.y, l);
      }
    }
    if (gl > 0.f) {
      const float wgt = ex2(gm - mx);
#pragma unroll
      for (int c = 0; c < DC; ++c) o[c] = fmaf(wgt, go[c], o[c]);
      l = fmaf(wgt, gl, l);
    }
  }
#pragma unroll
  for (int c = 0; c < DC; ++c) out[rh * DIM + c * D + t] = __float2bfloat16_rn(l > 0.f ? o[c] / l : 0.f);
}

// At head_dim 128 the combine keeps the compiler's own register choice (96); at head_dim 512 it is held to 128, so
// that one block fits on an SM beside the pass's CTA (168 x 288 registers) and attends its generated keys during the
// pass instead of after it (measured, config 3 at 8 x 512: 72.8 -> 61.7 us per layer).
__global__ void __launch_bounds__(128) combine_tc_kernel_d128(const Params p, int grid, __nv_bfloat16* __restrict__ out,
                                                              const GenKeys gen) {
  combine_tc_body<128>(p, grid, out, gen);
}
__global__ void __launch_bounds__(128, 4) combine_tc_kernel_d512(const Params p, int grid,
                                                                 __nv_bfloat16* __restrict__ out, const GenKeys gen) {
  combine_tc_body<512>(p, grid, out, gen);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  return fn;
}

bool make_cache_map(CUtensorMap* map, const void* base, int64_t rows, int heads, int64_t len, int64_t s_row,
                    int64_t s_head, int64_t s_pos, int dim, int box_rows = BN) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)dim, (cuuint64_t)len, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[3] = {(cuuint64_t)s_pos * 2, (cuuint64_t)s_head * 2, (cuuint64_t)s_row * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, OMNI_TC_L2_PROMOTION,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Queries [rows, heads, dim] as 16-row boxes of one head (dim / 64 boxes of 64 columns per unit), 128-byte swizzle.
bool make_query_map(CUtensorMap* map, const void* q, int64_t rows, int heads, int dim) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {(cuuint64_t)dim, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)dim * 2, (cuuint64_t)heads * dim * 2};
  cuuint32_t box[3] = {64, 1, (cuuint32_t)NQP};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(q), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace tcattn

bool tc_path_enabled(int dtype, int dim, int nq) {
  static const bool forced_off = [] {
    const char* e = getenv("OMNIASR_ATTN_PATH");
    return e && e[0] == 'c';  // "cuda_cores"
  }();
  return !forced_off && dtype == kBF16 && (dim == 128 || dim == 512) && nq >= 1 && nq <= tcattn::NQP &&
         tcattn::encode_fn() != nullptr;
}

int tc_segments(int64_t keys) { return (int)((keys + tcattn::BN - 1) / tcattn::BN) + 1; }

int tc_grid() { return device_sm_count(); }

// The pass instance's query columns for nq queries per unit (1, 2, 4, 8 or 16).
int tc_nqt(int nq) { return nq <= 1 ? 1 : nq <= 2 ? 2 : nq <= 4 ? 4 : nq <= 8 ? 8 : 16; }

// Tiles the producers prefetch into L2 ahead of their loads (OMNIASR_TC_PREFETCH overrides the default).
int tc_prefetch() {
  static const int n = [] {
    const char* e = getenv("OMNIASR_TC_PREFETCH");
    return e ? atoi(e) : 0;  // measured: prefetching past the ring only adds DRAM traffic
  }();
  return n < 0 ? 0 : n;
}

// Cost of a unit's start and epilogue in tile-eighths. Measured on B200 (config-2 and config-1 shapes, with the
// in-pass merge): units of several query rows split best at 10 (0.7 % faster than 8 on the verify step; 4-16
// swept), single-query units at 0 -- their epilogue is short, and a finer split evens out the CTAs' ends.
// OMNIASR_TC_UNIT_COST overrides both.
int tc_unit_cost(int nq) {
  static const int c = [] {
    const char* e = getenv("OMNIASR_TC_UNIT_COST");
    return e ? atoi(e) : -1;
  }();
  if (c >= 0) return c;
  return nq <= 1 ? 0 : 10;
}

int tc_prefill_segments(int batch, int heads, int width, int nq) {
  // The pass's own schedule (TileIter): unit (g, h) costs unit_cost + kTileCost * tiles at cost position pre(g) +
  // h * ucost(g); CTA b owns [b * per, (b + 1) * per). Group g = row * gpr + j covers queries 16j .. 16j + 15 and
  // reads min(16j + nq, width) keys.
  using namespace tcattn;
  const int gpr = (width + nq - 1) / nq;
  const int64_t ucost = tc_unit_cost(nq);
  auto cost = [&](int j) -> int64_t {
    const int64_t need = std::min<int64_t>((int64_t)j * nq + nq, width);
    const int64_t tiles = (need + BN - 1) / BN;
    return tiles > 0 ? ucost + kTileCost * tiles : 0;
  };
  int64_t total = 0;
  for (int j = 0; j < gpr; ++j) total += cost(j) * heads;
  total *= batch;
  const int grid = tc_grid();
  const int64_t per = std::max<int64_t>((total + grid - 1) / grid, kTileCost);
  int most = 1;
  int64_t pre = 0;
  for (int b = 0; b < batch; ++b)
    for (int j = 0; j < gpr; ++j) {
      const int64_t c = cost(j);
      const int64_t tiles = (c - ucost) / kTileCost;
      for (int h = 0; h < heads && tiles > 0; ++h) {
        const int64_t pos0 = pre + h * c + ucost;
        const int nseg = (int)((pos0 + kTileCost * (tiles - 1)) / per - pos0 / per + 1);
        most = std::max(most, nseg);
      }
      pre += c * heads;
    }
  return most;
}

size_t tc_prefill_workspace(int batch, int heads, int width, int dim, int nq) {
  const int st = tc_prefill_segments(batch, heads, width, nq);
  return kCounterBytes + partial_bytes((int64_t)tc_grid() * tcattn::NQP, 1, st, dim);
}

cudaError_t launch_tc_pass(const void* k, const void* v, int64_t cache_rows, int64_t cache_len, int64_t s_row,
                           int64_t s_head, int64_t s_pos, int keys, TcParams& p, cudaStream_t stream) {
  using namespace tcattn;
  if (p.dim != 128 && p.dim != 512) return cudaErrorInvalidValue;
  CUtensorMap kmap, vmap, kmap_half, vmap_half;
  CUtensorMap qmap;
  if (!make_cache_map(&kmap, k, cache_rows, p.heads, cache_len, s_row, s_head, s_pos, p.dim) ||
      !make_cache_map(&vmap, v, cache_rows, p.heads, cache_len, s_row, s_head, s_pos, p.dim) ||
      !make_cache_map(&kmap_half, k, cache_rows, p.heads, cache_len, s_row, s_head, s_pos, p.dim, 64) ||
      !make_cache_map(&vmap_half, v, cache_rows, p.heads, cache_len, s_row, s_head, s_pos, p.dim, 64) ||
      !make_query_map(&qmap, p.q, (int64_t)p.groups * p.nq, p.heads, p.dim))
    return cudaErrorInvalidValue;
  p.cap = cache_len < keys ? cache_len : keys;
  if (!p.prefill) p.st = tc_segments(keys);  // prefill mode: set by the caller (tc_prefill_segments)
  if (p.kv_div < 1) p.kv_div = 1;
  p.grid = tc_grid();
  p.unit_cost = tc_unit_cost(p.nq);
  p.prefetch = tc_prefetch();
  using Kern = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, Params);
  // head_dim 128: six 32 KB ring slots (three K and three V tiles in flight); head_dim 512: four (two chunks each),
  // as the query buffers and the stash grow four-fold.
  static const Kern table[2][5] = {
      {attn_tc_kernel<1, 6, 128>, attn_tc_kernel<2, 6, 128>, attn_tc_kernel<4, 6, 128>, attn_tc_kernel<8, 6, 128>,
       attn_tc_kernel<16, 6, 128>},
      {attn_tc_kernel<1, 4, 512>, attn_tc_kernel<2, 4, 512>, attn_tc_kernel<4, 4, 512>, attn_tc_kernel<8, 4, 512>,
       attn_tc_kernel<16, 4, 512>}};
  const int di = p.dim == 128 ? 0 : 1;
  const int ci = p.nq <= 1 ? 0 : p.nq <= 2 ? 1 : p.nq <= 4 ? 2 : p.nq <= 8 ? 3 : 4;
  const Kern kern = table[di][ci];
  const int bytes = di == 0 ? Smem<6, 128>::BYTES : Smem<4, 512>::BYTES;
  static bool configured[2][5] = {};
  if (!configured[di][ci]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    configured[di][ci] = true;
  }
  // Programmatic dependent launch: the set-up above griddepcontrol.wait overlaps the previous kernel.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)p.grid);
  cfg.blockDim = dim3(threads_for(p.dim, tc_nqt(p.nq)));
  cfg.dynamicSmemBytes = (size_t)bytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, kmap, vmap, qmap, kmap_half, vmap_half, p);
}

cudaError_t launch_tc_combine(const TcParams& p, void* out, const GenKeys& gen, cudaStream_t stream) {
  using namespace tcattn;
  // Programmatic dependent launch: the combine's blocks start (and compute their unit's place) while the pass
  // drains, and wait for it (griddepcontrol.wait) before reading its partials.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((int64_t)p.groups * p.nq * p.heads));
  cfg.blockDim = dim3(128);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out);
  auto kern = p.dim == 512 ? combine_tc_kernel_d512 : combine_tc_kernel_d128;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p, p.grid, o, gen);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();  // no programmatic launch here: an ordinary one
    kern<<<cfg.gridDim, cfg.blockDim, 0, stream>>>(p, p.grid, o, gen);
    e = cudaGetLastError();
  }
  return e;
}

}  // namespace omni
