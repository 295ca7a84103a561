// Split-KV attention over a bf16 KV cache on the 5th-generation tensor cores (tcgen05 + TMEM), head_dim 128,
// up to 16 queries per group (decode: 1, draft verify: 1 + k, beam context: beams).
//
// Schedule (persistent, stream-K): the keys of every (group, head) unit are cut into 128-key tiles; the grid is
// one CTA per SM and CTA b takes the contiguous tile range [b * per, (b + 1) * per) of the concatenated units, so
// every SM streams the same number of K/V bytes whatever the ragged lengths. A unit cut between CTAs leaves one
// partial (max, sum, unnormalised output) per CTA ("segment"); the combine kernel merges the segments of a unit.
//
// One CTA: warp 4 is the TMA producer (K and V tiles, two 64-column boxes each, 128-byte swizzle, into a ring of
// six 32 KB slots: three tiles in flight); warps 0-3 are the consumers, thread t owning TMEM lane t:
//   S^T[128 keys x 16 q]  = K_tile [128 x 128] . Q^T         (tcgen05.mma, M=128 N=16, K-major A and B)
//   softmax over the keys of each query column (online, fp32, log2 units), P^T written to shared memory (bf16)
//   O^T[128 dims x 16 q]  = V_tile^T [128 x 128 keys] . P^T   (M=128 N=16, MN-major A and B)
// The per-tile O^T is read back from TMEM and accumulated in registers (thread t = head dim t).
//
// Algorithm of the reference restated: omniasr_trt/kernels.py:56-113 (_beam_ctx, CAUSAL for drafts) and
// kernels.py:163-195 (_attn_split): the same online softmax per split, merged by the combine
// (kernels.py:146-161 / :197-211).

#include <cudaTypedefs.h>
#include <math.h>
#include <stdlib.h>

#include "attention.cuh"
#include "tc.cuh"

namespace omni {

namespace tcattn {

constexpr int D = 128;
constexpr int BN = 128;          // keys per tile (the MMA's M)
constexpr int NQP = 16;          // query columns (the MMA's N)
constexpr int SLOTS = 6;         // ring slots: K and V of 3 tiles
constexpr int SLOT_BYTES = BN * D * 2;
constexpr int BOX_BYTES = BN * 64 * 2;  // one 64-column box of a tile
constexpr int Q_OFF = SLOTS * SLOT_BYTES;
constexpr int P_OFF = Q_OFF + NQP * D * 2;
constexpr int RED_OFF = P_OFF + 2 * NQP * BN * 2;
constexpr int SMEM_BYTES = RED_OFF + 4 * NQP * 4 + 1024;  // + alignment slack
constexpr int THREADS = 160;
constexpr uint32_t TMEM_COLS = 64;  // S^T x2 (cols 0-31), O^T x2 (cols 32-63)
constexpr uint32_t IDESC_S = idesc_bf16(128, NQP, 0, 0);
constexpr uint32_t IDESC_O = idesc_bf16(128, NQP, 1, 1);

using Params = TcParams;

// Keys unit (g, .) must read, clamped to the cache and the key bound.
OMNI_DEV int64_t unit_need(const Params& p, int g) {
  int64_t n = p.lengths[g] + (p.causal ? p.nq - 1 : 0);
  n = n < 0 ? 0 : n;
  return n > p.cap ? p.cap : n;
}

// Walks the global tile sequence (groups outer, heads inner, tiles of a unit innermost).
struct Walk {
  int g;
  int64_t pre;    // first global tile of group g
  int64_t tiles;  // tiles per unit of group g
  int64_t need;   // keys per unit of group g
  OMNI_DEV void start(const Params& p, int64_t x) {
    g = 0;
    pre = 0;
    for (;;) {
      need = unit_need(p, g);
      tiles = (need + BN - 1) / BN;
      if (g == p.groups - 1 || x < pre + tiles * p.heads) break;
      pre += tiles * p.heads;
      ++g;
    }
  }
  // Moves forward to the group holding global tile x (x never decreases).
  OMNI_DEV void seek(const Params& p, int64_t x) {
    while (x >= pre + tiles * p.heads && g < p.groups - 1) {
      pre += tiles * p.heads;
      ++g;
      need = unit_need(p, g);
      tiles = (need + BN - 1) / BN;
    }
  }
};

OMNI_DEV int64_t total_tiles(const Params& p) {
  int64_t t = 0;
  for (int g = 0; g < p.groups; ++g) t += (unit_need(p, g) + BN - 1) / BN * p.heads;
  return t;
}

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

constexpr float kRescale = 8.f;  // log2 units: probabilities may reach 2^8 before the running max is raised

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

// S^T[buf] = K_tile (slot ks) . Q^T  (thread 0).
OMNI_DEV void issue_scores(uint32_t tbase, int buf, const unsigned char* kslot, const unsigned char* qs) {
  const uint32_t kaddr = smem_addr(kslot);
  const uint32_t qaddr = smem_addr(qs);
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint64_t a = smem_desc(kaddr + (kk >> 2) * BOX_BYTES + (kk & 3) * 32, 16, 1024, kLayoutSw128);
    const uint64_t b = smem_desc(qaddr + kk * 256, 128, 2048, kLayoutNone);
    mma_bf16_ss(tbase + buf * NQP, a, b, IDESC_S, kk > 0 ? 1u : 0u);
  }
}

// O^T[buf] = V_tile^T (slot vs) . P^T[buf]  (thread 0).
OMNI_DEV void issue_values(uint32_t tbase, int buf, const unsigned char* vslot, const unsigned char* pbuf) {
  const uint32_t vaddr = smem_addr(vslot);
  const uint32_t paddr = smem_addr(pbuf);
#pragma unroll
  for (int kk = 0; kk < BN / 16; ++kk) {
    const uint64_t a = smem_desc(vaddr + kk * 2048, BOX_BYTES, 1024, kLayoutSw128);
    const uint64_t b = smem_desc(paddr + kk * 256, 128, 2048, kLayoutNone);
    mma_bf16_ss(tbase + 2 * NQP + buf * NQP, a, b, IDESC_O, kk > 0 ? 1u : 0u);
  }
}

// NQT: query columns processed (a compile-time bound >= nq; the MMA always computes 16).
template <int NQT>
__global__ void __launch_bounds__(THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                   const Params p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[SLOTS], empty[SLOTS], bar_s[2], bar_o[2], drain;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ volatile int issued_k, issued_v, done_tiles;  // K / V loads issued, tiles fully consumed

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const int64_t total = total_tiles(p);
  const int64_t per = total > 0 ? (total + gridDim.x - 1) / gridDim.x : 1;
  const int64_t x0 = (int64_t)blockIdx.x * per;
  const int64_t x1 = min(total, x0 + per);
  if (x0 >= x1) return;  // nothing for this CTA (uniform)

  if (tid == 0) {
    for (int s = 0; s < SLOTS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar_s[s], 1);
      mbar_init(&bar_o[s], 1);
    }
    mbar_init(&drain, 1);
    mbar_fence_init();
    abort_flag = 0;
    issued_k = issued_v = done_tiles = 0;
  }
  if (warp == 0) tmem_alloc(&tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = tmem_base;

  if (warp == 4) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tmap(&kmap);
      prefetch_tmap(&vmap);
      Walk w;
      w.start(p, x0);
      for (int64_t x = x0; x < x1; ++x) {
        if (abort_flag) break;
        w.seek(p, x);
        const int64_t r = x - w.pre;
        const int h = (int)(r / w.tiles);
        const int k0 = (int)(r % w.tiles) * BN;
        const int it = (int)(x - x0);
        const int ks = 2 * (it % 3), vs = ks + 1;
        const int use = it / 3;
        if (use >= 1 && !mbar_wait(&empty[ks], (use - 1) & 1)) {
          abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[ks], SLOT_BYTES);
        tma_load_4d(smem + ks * SLOT_BYTES, &kmap, 0, k0, h, w.g, &full[ks]);
        tma_load_4d(smem + ks * SLOT_BYTES + BOX_BYTES, &kmap, 64, k0, h, w.g, &full[ks]);
        issued_k = it + 1;
        if (use >= 1 && !mbar_wait(&empty[vs], (use - 1) & 1)) {
          abort_flag = 1;
          break;
        }
        mbar_arrive_expect_tx(&full[vs], SLOT_BYTES);
        tma_load_4d(smem + vs * SLOT_BYTES, &vmap, 0, k0, h, w.g, &full[vs]);
        tma_load_4d(smem + vs * SLOT_BYTES + BOX_BYTES, &vmap, 64, k0, h, w.g, &full[vs]);
        issued_v = it + 1;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ consumers (128 threads)
    // Per tile: S^T (issued one tile ahead) -> softmax (the running max is raised only when a score passes it by
    // 2^8, so the cross-thread max is rare) -> P^T -> O^T (accumulated one tile later, overlapping the next tile).
    const uint32_t lane_off = (uint32_t)(32 * warp) << 16;
    unsigned char* qs = smem + Q_OFF;
    float* red = reinterpret_cast<float*>(smem + RED_OFF);
    Walk w;
    w.start(p, x0);
    float m[NQT], lpart[NQT], acc[NQT], scl[NQT];
    int lim[NQT];
    int g = 0, h = 0;
    int64_t unit_first = 0;
    bool pending = false;  // an O^T tile issued and not yet accumulated
    bool ok_all = true;
    int it = 0;
    for (int64_t x = x0; x < x1; ++x, ++it) {
      w.seek(p, x);
      const int64_t r = x - w.pre;
      const int tt = (int)(r % w.tiles);
      const int buf = it & 1;
      const int ks = 2 * (it % 3), vs = ks + 1;
      const uint32_t slot_parity = (it / 3) & 1;
      const uint32_t buf_parity = (it >> 1) & 1;
      const bool first = tt == 0 || x == x0;
      const bool last = tt == w.tiles - 1 || x == x1 - 1;
      if (first) {
        g = w.g;
        h = (int)(r / w.tiles);
        unit_first = w.pre + (int64_t)h * w.tiles;
        const int64_t n = p.lengths[g];
#pragma unroll
        for (int j = 0; j < NQT; ++j) {
          int64_t lj = n + (p.causal ? j : 0);
          lj = lj < 0 ? 0 : lj;
          lim[j] = j < p.nq ? (int)(lj > w.need ? w.need : lj) : 0;
          m[j] = -INFINITY;
          lpart[j] = 0.f;
          acc[j] = 0.f;
        }
        for (int i = tid; i < NQP * (D / 8); i += 128) {
          const int j = i / (D / 8), c = i % (D / 8);
          uint4 val = make_uint4(0u, 0u, 0u, 0u);
          if (j < p.nq)
            val = __ldg(reinterpret_cast<const uint4*>(p.q + (((int64_t)g * p.nq + j) * p.heads + h) * D) + c);
          *reinterpret_cast<uint4*>(qs + (j >> 3) * 2048 + c * 128 + (j & 7) * 16) = val;
        }
        fence_async_smem();
        __syncwarp();
        named_sync(1, 128);
        if (tid == 0) {
          if (mbar_wait(&full[ks], slot_parity)) {
            tc_fence_after();
            issue_scores(tbase, buf, smem + ks * SLOT_BYTES, qs);
            tc_commit(&bar_s[buf]);
            tc_commit(&empty[ks]);
          } else {
            abort_flag = 1;
          }
        }
      }
      const int key = tt * BN + tid;

      // Scores of this tile.
      if (!mbar_wait(&bar_s[buf], buf_parity)) abort_flag = 1;
      tc_fence_after();
      __syncwarp();
      float s[NQP];
      tmem_ld16(tbase + lane_off + buf * NQP, s);
      float xv[NQT];
      bool over = false;
#pragma unroll
      for (int j = 0; j < NQT; ++j) {
        xv[j] = key < lim[j] ? s[j] * p.qscale : -INFINITY;
        over |= xv[j] > m[j] + kRescale;
      }
      const bool any_over = named_sync_or(1, 128, over);
      if (abort_flag) {  // uniform: written before the barrier
        ok_all = false;
        break;
      }
      if (any_over) {
        // Raise the running max of every column to this tile's maximum (cross-thread reduction).
#pragma unroll
        for (int j = 0; j < NQT; ++j) {
          float v = xv[j];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
          if (lane == 0) red[warp * NQP + j] = v;
        }
        named_sync(1, 128);
#pragma unroll
        for (int j = 0; j < NQT; ++j) {
          const float tmax = fmaxf(fmaxf(red[j], red[NQP + j]), fmaxf(red[2 * NQP + j], red[3 * NQP + j]));
          const float mnew = fmaxf(m[j], tmax);
          scl[j] = ex2(m[j] - (mnew == -INFINITY ? 0.f : mnew));  // 0 while the column has seen no key
          m[j] = mnew;
          acc[j] *= scl[j];
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
        pr[j] = ex2(xv[j] - (m[j] == -INFINITY ? 0.f : m[j]));
        lpart[j] += pr[j];
      }
      {
        unsigned char* pb = smem + P_OFF + buf * (NQP * BN * 2);
        uint32_t wv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(pr[2 * i]));
          const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(pr[2 * i + 1]));
          wv[i] = lo | (hi << 16);
        }
        *reinterpret_cast<uint4*>(pb + tid * 16) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
        if (NQT > 8) *reinterpret_cast<uint4*>(pb + 2048 + tid * 16) = make_uint4(wv[4], wv[5], wv[6], wv[7]);
        else *reinterpret_cast<uint4*>(pb + 2048 + tid * 16) = make_uint4(0u, 0u, 0u, 0u);
      }
      // A tile that ends inside the unit's keys: zero the V rows past them (they may hold anything).
      const bool partial = (int64_t)tt * BN + BN > w.need;
      if (partial) {
        if (!mbar_wait(&full[vs], slot_parity)) abort_flag = 1;
        if (key >= w.need) {
          unsigned char* row = smem + vs * SLOT_BYTES + tid * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            *reinterpret_cast<uint4*>(row + c * 16) = make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4*>(row + BOX_BYTES + c * 16) = make_uint4(0u, 0u, 0u, 0u);
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncwarp();
      named_sync(1, 128);  // P^T (and zeroed V rows) ready

      if (tid == 0) {
        tc_fence_after();
        if (partial || mbar_wait(&full[vs], slot_parity)) {
          issue_values(tbase, buf, smem + vs * SLOT_BYTES, smem + P_OFF + buf * (NQP * BN * 2));
          tc_commit(&bar_o[buf]);
          tc_commit(&empty[vs]);
        } else {
          abort_flag = 1;
        }
        if (!last) {  // the next tile belongs to this unit: its scores now, overlapping this tile's tail
          const int ks2 = 2 * ((it + 1) % 3);
          if (mbar_wait(&full[ks2], ((it + 1) / 3) & 1)) {
            issue_scores(tbase, buf ^ 1, smem + ks2 * SLOT_BYTES, qs);
            tc_commit(&bar_s[buf ^ 1]);
            tc_commit(&empty[ks2]);
          } else {
            abort_flag = 1;
          }
        }
      }
      __syncwarp();

      // The previous tile's O^T, brought to this tile's max.
      if (pending) {
        if (!mbar_wait(&bar_o[buf ^ 1], ((it - 1) >> 1) & 1)) abort_flag = 1;
        tc_fence_after();
        __syncwarp();
        float o[NQP];
        tmem_ld16(tbase + lane_off + 2 * NQP + (buf ^ 1) * NQP, o);
#pragma unroll
        for (int j = 0; j < NQT; ++j) acc[j] = fmaf(scl[j], o[j], acc[j]);
        if (tid == 0) done_tiles = it;
      }
      pending = true;

      if (last) {
        // End of this CTA's part of the unit: this tile's O^T, then the unit's segment (or its output).
        if (!mbar_wait(&bar_o[buf], buf_parity)) abort_flag = 1;
        tc_fence_after();
        __syncwarp();
        float o[NQP];
        tmem_ld16(tbase + lane_off + 2 * NQP + buf * NQP, o);
#pragma unroll
        for (int j = 0; j < NQT; ++j) acc[j] += o[j];
        pending = false;
        if (tid == 0) done_tiles = it + 1;
#pragma unroll
        for (int j = 0; j < NQT; ++j) {
          float v = lpart[j];
#pragma unroll
          for (int o2 = 16; o2 > 0; o2 >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o2);
          if (lane == 0) red[warp * NQP + j] = v;
        }
        named_sync(1, 128);
        const int seg = (int)(blockIdx.x - unit_first / per);
        const bool whole = (unit_first + w.tiles - 1) / per == unit_first / per;
#pragma unroll
        for (int j = 0; j < NQT; ++j) {
          if (j < p.nq) {
            const float l = red[j] + red[NQP + j] + red[2 * NQP + j] + red[3 * NQP + j];
            const int64_t rowh = ((int64_t)g * p.nq + j) * p.heads + h;
            if (whole && p.out) {
              p.out[rowh * D + tid] = __float2bfloat16_rn(l > 0.f ? acc[j] / l : 0.f);
            } else {
              const int64_t part = rowh * p.st + seg;
              p.part_o[part * D + tid] = acc[j];
              if (tid == 0) reinterpret_cast<float2*>(p.part_ml)[part] = make_float2(m[j], l);
            }
          }
        }
        named_sync(1, 128);
      }
      tc_fence_before();
    }
    if (!ok_all) abort_flag = 1;
  }
  __syncthreads();
  if (abort_flag && tid == 0) {
    raise_status(p.status, kStatusTimeout);
    tc_commit(&drain);  // every MMA thread 0 issued has completed once this arrives
    mbar_wait(&drain, 0);
    // Let TMA loads that were issued but not consumed land before the CTA's shared memory goes away (at most
    // three tiles are in flight, so each slot appears once in these windows).
    for (int i = done_tiles; i < issued_k; ++i) mbar_wait(&full[2 * (i % 3)], (i / 3) & 1);
    for (int i = done_tiles; i < issued_v; ++i) mbar_wait(&full[2 * (i % 3) + 1], (i / 3) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

// Merges the segments of each (query row, head): out = sum w_s o_s / sum w_s l_s, plus (beam search) the splits
// of a second partial region. A unit the pass finished inside one CTA was written by the pass itself.
__global__ void __launch_bounds__(128) combine_tc_kernel(const Params p, int grid, __nv_bfloat16* __restrict__ out,
                                                         const float* __restrict__ extra_o,
                                                         const float* __restrict__ extra_ml, int extra_st) {
  __shared__ long long red_total[4], red_pre[4];
  __shared__ long long unit_tiles;
  const int64_t rh = blockIdx.x;
  const int row = (int)(rh / p.heads);
  const int h = (int)(rh % p.heads);
  const int g = row / p.nq;
  const int t = threadIdx.x;
  long long tot = 0, pre = 0;
  for (int i = t; i < p.groups; i += 128) {
    const long long n = (unit_need(p, i) + BN - 1) / BN;
    tot += n * p.heads;
    if (i < g) pre += n * p.heads;
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
  const long long start = red_pre[0] + red_pre[1] + red_pre[2] + red_pre[3] + (long long)h * tiles;
  if (t == 0 && h == 0 && row % p.nq == 0) {
    const int64_t raw = p.lengths[g] + (p.causal ? p.nq - 1 : 0);
    if (p.lengths[g] < 0 || raw > p.cap) raise_status(p.status, kStatusIndex);
  }
  const long long per = total > 0 ? (total + grid - 1) / grid : 1;
  const int nseg = tiles > 0 ? (int)((start + tiles - 1) / per - start / per + 1) : 0;
  if (nseg == 1 && extra_ml == nullptr && p.out != nullptr) return;  // finished by the pass
  const float2* ml = reinterpret_cast<const float2*>(p.part_ml) + rh * p.st;
  const float2* ml2 = extra_ml ? reinterpret_cast<const float2*>(extra_ml) + rh * extra_st : nullptr;
  float mx = -INFINITY;
  for (int s = 0; s < nseg; ++s) mx = fmaxf(mx, ml[s].x);
  for (int s = 0; ml2 && s < extra_st; ++s) mx = fmaxf(mx, ml2[s].x);
  float o = 0.f, l = 0.f;
  if (mx != -INFINITY) {
    for (int s = 0; s < nseg; ++s) {
      const float2 e = ml[s];
      if (e.x != -INFINITY) {
        const float wgt = ex2(e.x - mx);
        o = fmaf(wgt, p.part_o[(rh * p.st + s) * D + t], o);
        l = fmaf(wgt, e.y, l);
      }
    }
    for (int s = 0; ml2 && s < extra_st; ++s) {
      const float2 e = ml2[s];
      if (e.x != -INFINITY) {
        const float wgt = ex2(e.x - mx);
        o = fmaf(wgt, extra_o[(rh * extra_st + s) * D + t], o);
        l = fmaf(wgt, e.y, l);
      }
    }
  }
  out[rh * D + t] = __float2bfloat16_rn(l > 0.f ? o / l : 0.f);
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
                    int64_t s_head, int64_t s_pos) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)len, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[3] = {(cuuint64_t)s_pos * 2, (cuuint64_t)s_head * 2, (cuuint64_t)s_row * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)BN, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
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
  return !forced_off && dtype == kBF16 && dim == tcattn::D && nq >= 1 && nq <= tcattn::NQP &&
         tcattn::encode_fn() != nullptr;
}

int tc_segments(int64_t keys) { return (int)((keys + tcattn::BN - 1) / tcattn::BN) + 1; }

int tc_grid() { return device_sm_count(); }

cudaError_t launch_tc_pass(const void* k, const void* v, int64_t cache_rows, int64_t cache_len, int64_t s_row,
                           int64_t s_head, int64_t s_pos, int keys, TcParams& p, cudaStream_t stream) {
  using namespace tcattn;
  CUtensorMap kmap, vmap;
  if (!make_cache_map(&kmap, k, cache_rows, p.heads, cache_len, s_row, s_head, s_pos) ||
      !make_cache_map(&vmap, v, cache_rows, p.heads, cache_len, s_row, s_head, s_pos))
    return cudaErrorInvalidValue;
  p.cap = cache_len < keys ? cache_len : keys;
  p.st = tc_segments(keys);
  p.grid = tc_grid();
  auto kern = p.nq <= 1 ? attn_tc_kernel<1> : p.nq <= 2 ? attn_tc_kernel<2> : p.nq <= 4 ? attn_tc_kernel<4>
            : p.nq <= 8 ? attn_tc_kernel<8> : attn_tc_kernel<16>;
  static bool configured[5] = {false, false, false, false, false};
  const int ci = p.nq <= 1 ? 0 : p.nq <= 2 ? 1 : p.nq <= 4 ? 2 : p.nq <= 8 ? 3 : 4;
  if (!configured[ci]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured[ci] = true;
  }
  kern<<<p.grid, THREADS, SMEM_BYTES, stream>>>(kmap, vmap, p);
  return cudaGetLastError();
}

cudaError_t launch_tc_combine(const TcParams& p, void* out, const float* extra_o, const float* extra_ml, int extra_st,
                              cudaStream_t stream) {
  using namespace tcattn;
  combine_tc_kernel<<<(unsigned)((int64_t)p.groups * p.nq * p.heads), 128, 0, stream>>>(
      p, p.grid, reinterpret_cast<__nv_bfloat16*>(out), extra_o, extra_ml, extra_st);
  return cudaGetLastError();
}

}  // namespace omni
