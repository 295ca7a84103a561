// Causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), bf16, head_dim 512 -- the shipped
// omniASR-LLM decoder's 8 heads x 512 (omniasr_trt/modeling.py:30-35).
//
// out[b, w, h] = softmax(q[b, h, w] . k[b, h, :w+1]^T * scale) . v[b, h, :w+1]   for w < W
// (F.scaled_dot_product_attention(q, k, v, is_causal=True) of the reference's prefill, decode.py:171).
//
// The head_dim-128 kernel (prefill.cu) keeps a 128 x 128 fp32 accumulator per query tile in TMEM; at head_dim 512
// the accumulator alone (128 x 512 fp32) fills all of TMEM, and one query tile is 128 KB of shared memory. So a unit
// (row b, head h, 128-query tile qt) runs as two passes over its key tiles, pass p accumulating head dims
// 256p .. 256p + 255 of O: both passes form the same scores S = Q K^T over all 512 dims (four 128-dim chunks
// accumulated in TMEM) and the same probabilities; the second pass recomputes them (one and a half times the
// minimum MMA work) instead of storing them. The work is MMA-bound at this head_dim: a tile pass is 32 SS MMAs
// (128 x 128 x 16) for S and 32 TS MMAs (128 x 64 x 16) for P V, against one softmax of a 128 x 128 tile.
//
// Shared memory (224 KB): the unit's query tile as four 128-dim chunks (loaded once for both passes; chunk c is
// refilled with the next unit's as soon as the last S MMA that reads it has completed), a 2-slot ring of 128-dim K
// chunks, a 2-slot ring of 64-dim V sub-chunks (128 keys each; 128-byte swizzle throughout).
// TMEM (512 columns): S double-buffered at [0, 128) and [128, 256), O of the pass's 256 dims at [256, 512); P (bf16
// pairs) over S, read by the A-from-TMEM MMA.
// Roles (512 threads), as in prefill.cu: warp 12 K chunk loads, warp 14 V sub-chunk loads, warp 13 S MMAs, warp 15
// P V MMAs, warps 0-3 / 4-7 softmax warpgroups (thread = query row, warpgroup x the keys 64x .. 64x + 63 of every
// tile, one running max per row shared through a barrier per tile), warps 8-11 the epilogue (and the query loads,
// by its first thread).

#include <cudaTypedefs.h>
#include <math.h>

#include "attention.cuh"
#include "prefill.cuh"
#include "prefill_common.cuh"

namespace omni {
namespace prefillw {

using namespace pfx;

constexpr int D = 512;
constexpr int DC = D / 128;        // 128-dim chunks of Q and K
constexpr int DH = D / 2;          // head dims of O per pass
constexpr int NSUB = DH / 64;      // 64-dim V sub-chunks per pass
constexpr int BM = 128;            // queries per tile
constexpr int BN = 128;            // keys per tile
constexpr int CHUNK = BN * 128 * 2;  // 128 rows x 128 dims
constexpr int BOX = BN * 64 * 2;     // 128 rows x 64 dims: one TMA box
constexpr int KS = 2, VS = 2;
constexpr int Q_OFF = 0;
constexpr int K_OFF = Q_OFF + DC * CHUNK;
constexpr int V_OFF = K_OFF + KS * CHUNK;
constexpr int SMEM_BYTES = V_OFF + VS * BOX;
constexpr int NSB = 2;
constexpr int NWG = 2;
constexpr int KW = BN / NWG;  // keys per softmax warpgroup
constexpr int DW = DH / NWG;  // head dims of O each softmax warpgroup rescales
constexpr int W_EPI = 4 * NWG, W_LOADK = W_EPI + 4, W_MMA = W_LOADK + 1, W_LOADV = W_LOADK + 2, W_MMA_PV = W_LOADK + 3;
constexpr int THREADS = 32 * (W_MMA_PV + 1);
constexpr int SM_THREADS = 128 * NWG;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S = 0, COL_O = NSB * 128;
constexpr uint32_t IDESC_S = idesc_bf16(BM, BN, 0, 0);
constexpr uint32_t IDESC_O = idesc_bf16(BM, 64, 0, 1);
constexpr float kRescale = 8.f;
constexpr int kPolyEvery = 4;  // probabilities of one pair in this many by ex2_fma

struct Params {
  int batch, heads, width, qtiles;
  int group;
  float qscale;  // scale * log2(e)
  __nv_bfloat16* out;
  int64_t out_sb, out_sw, out_sh;
  int* status;
};

struct alignas(1024) Ctl {
  uint64_t k_full[KS], k_empty[KS], v_full[VS], v_empty[VS], q_full[DC], q_empty[DC];
  uint64_t s_full[NSB], pv_done[NSB], p_full[NWG][NSB];
  uint64_t o_ready, o_free, l_full, l_free, drain;
  float tmax[NWG][BM];
  float lsum[NWG][BM];
  uint32_t tmem_base;
  int abort_flag, issued_k, issued_v, issued_q;
};
static_assert(sizeof(Ctl) + SMEM_BYTES <= 232448, "shared memory per block");
static_assert(NSB * 128 + DH <= TMEM_COLS, "S buffers and O in TMEM");

__global__ void __launch_bounds__(THREADS, 1)
    prefill_wide_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const Params p, const __grid_constant__ Sched sched) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ Ctl ctl;
  uint64_t *k_full = ctl.k_full, *k_empty = ctl.k_empty, *v_full = ctl.v_full, *v_empty = ctl.v_empty;
  uint64_t *q_full = ctl.q_full, *q_empty = ctl.q_empty, *s_full = ctl.s_full, *pv_done = ctl.pv_done;
  uint64_t(*p_full)[NSB] = ctl.p_full;
  uint64_t &o_ready = ctl.o_ready, &o_free = ctl.o_free, &l_full = ctl.l_full, &l_free = ctl.l_free;
  uint64_t& drain = ctl.drain;
  volatile int& abort_flag = ctl.abort_flag;
  volatile int &issued_k = ctl.issued_k, &issued_v = ctl.issued_v, &issued_q = ctl.issued_q;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int units = p.batch * p.heads * p.qtiles;
  if ((int)blockIdx.x >= units) return;
  if (smem_addr(smem) & 1023u) {
    if (tid == 0) raise_status(p.status, kStatusLayout);
    return;
  }
  if (tid == 0) {
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int c = 0; c < DC; ++c) {
      mbar_init(&q_full[c], 1);
      mbar_init(&q_empty[c], 1);
    }
    for (int j = 0; j < NSB; ++j) {
      mbar_init(&s_full[j], 1);
      mbar_init(&pv_done[j], 1);
      for (int x = 0; x < NWG; ++x) mbar_init(&p_full[x][j], 128);
    }
    mbar_init(&o_ready, 1);
    mbar_init(&o_free, 128);
    mbar_init(&l_full, SM_THREADS);
    mbar_init(&l_free, 128);
    mbar_init(&drain, 2);
    mbar_fence_init();
    abort_flag = 0;
    issued_k = issued_v = issued_q = 0;
  }
  if (warp == W_EPI) tmem_alloc(&ctl.tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dependency_wait();  // q, k, v may come from the kernel before (launched as a programmatic dependent)
  const uint32_t tbase = ctl.tmem_base;
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (mbar_wait_or(bar, parity, &abort_flag)) return true;
    abort_flag = 1;
    return false;
  };
  auto decode = [&](int u, int& b, int& h, int& qt) { unit_of(p.batch, p.heads, p.qtiles, p.group, u, b, h, qt); };

  if (warp == W_LOADK) {
    // ------------------------------------------------------------------ K: chunk c of key tile kt, both passes
    if (lane == 0) {
      prefetch_tmap(&kmap);
      int kc = 0;
      for (int n = 0, u; (u = cta_unit(sched, units, n)) >= 0 && !abort_flag; ++n) {
        int b, h, qt;
        decode(u, b, h, qt);
        for (int pass = 0; pass < 2 && !abort_flag; ++pass)
          for (int kt = 0; kt <= qt && !abort_flag; ++kt)
            for (int c = 0; c < DC && !abort_flag; ++c, ++kc) {
              const int slot = kc % KS, use = kc / KS;
              if (use >= 1 && !wait(&k_empty[slot], (use - 1) & 1)) break;
              mbar_arrive_expect_tx(&k_full[slot], CHUNK);
              unsigned char* dst = smem + K_OFF + slot * CHUNK;
              tma_load_4d(dst, &kmap, c * 128, kt * BN, h, b, &k_full[slot]);
              tma_load_4d(dst + BOX, &kmap, c * 128 + 64, kt * BN, h, b, &k_full[slot]);
              issued_k = kc + 1;
            }
      }
    }
    __syncwarp();
  } else if (warp == W_LOADV) {
    // ------------------------------------------------------------------ V: the pass's 64-dim sub-chunks of tile kt
    if (lane == 0) {
      prefetch_tmap(&vmap);
      int vc = 0;
      for (int n = 0, u; (u = cta_unit(sched, units, n)) >= 0 && !abort_flag; ++n) {
        int b, h, qt;
        decode(u, b, h, qt);
        for (int pass = 0; pass < 2 && !abort_flag; ++pass)
          for (int kt = 0; kt <= qt && !abort_flag; ++kt)
            for (int sc = 0; sc < NSUB && !abort_flag; ++sc, ++vc) {
              const int slot = vc % VS, use = vc / VS;
              if (use >= 1 && !wait(&v_empty[slot], (use - 1) & 1)) break;
              mbar_arrive_expect_tx(&v_full[slot], BOX);
              tma_load_4d(smem + V_OFF + slot * BOX, &vmap, pass * DH + sc * 64, kt * BN, h, b, &v_full[slot]);
              issued_v = vc + 1;
            }
      }
    }
    __syncwarp();
  } else if (warp == W_MMA) {
    // ------------------------------------------------------------------ S[t % NSB] = sum over chunks Q_c K_c(t)^T
    if (lane == 0) {
      const uint64_t kdesc0 = smem_desc(smem_addr(smem + K_OFF), 16, 1024, kLayoutSw128);
      const uint64_t qdesc0 = smem_desc(smem_addr(smem + Q_OFF), 16, 1024, kLayoutSw128);
      int tile = 0, kc = 0;
      bool ok = true;
      for (int n = 0, u; (u = cta_unit(sched, units, n)) >= 0 && ok && !abort_flag; ++n) {
        int b, h, qt;
        decode(u, b, h, qt);
        for (int pass = 0; pass < 2 && ok; ++pass) {
          for (int kt = 0; kt <= qt && ok; ++kt, ++tile) {
            const int sb = tile % NSB;
            if (tile >= NSB && !wait(&pv_done[sb], ((tile - NSB) / NSB) & 1)) {
              ok = false;
              break;
            }
            const uint32_t dcol = tbase + COL_S + sb * 128;
            for (int c = 0; c < DC; ++c, ++kc) {
              if (pass == 0 && kt == 0 && !wait(&q_full[c], n & 1)) {
                ok = false;
                break;
              }
              const int slot = kc % KS;
              if (!wait(&k_full[slot], (kc / KS) & 1)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t qd = qdesc0 + (uint64_t)(c * (CHUNK >> 4));
              const uint64_t kd = kdesc0 + (uint64_t)(slot * (CHUNK >> 4));
#pragma unroll
              for (int kk = 0; kk < 8; ++kk) {
                const uint64_t off = (uint64_t)((((kk >> 2) * BOX + (kk & 3) * 32) >> 4));
                mma_bf16_ss(dcol, qd + off, kd + off, IDESC_S, (c > 0 || kk > 0) ? 1u : 0u);
              }
              tc_commit(&k_empty[slot]);
              if (pass == 1 && kt == qt) tc_commit(&q_empty[c]);  // the unit's last read of query chunk c
            }
            if (!ok) break;
            tc_commit(&s_full[sb]);
          }
        }
      }
      if (!ok) abort_flag = 1;
    }
    __syncwarp();
  } else if (warp == W_MMA_PV) {
    // ------------------------------------------------------------------ O[:, 64 sc ..] += P(t) V(t)[:, sc]
    if (lane == 0) {
      const uint64_t vdesc0 = smem_desc(smem_addr(smem + V_OFF), BOX, 1024, kLayoutSw128);
      int tile = 0, vc = 0, item = 0;
      bool ok = true;
      for (int n = 0, u; (u = cta_unit(sched, units, n)) >= 0 && ok && !abort_flag; ++n) {
        int b, h, qt;
        decode(u, b, h, qt);
        for (int pass = 0; pass < 2 && ok; ++pass, ++item) {
          for (int kt = 0; kt <= qt && ok; ++kt, ++tile) {
            const int pb = tile % NSB, pu = tile / NSB;
            if (kt == 0 && item >= 1 && !wait(&o_free, (item - 1) & 1)) {
              ok = false;
              break;
            }
            for (int x = 0; x < NWG && ok; ++x) ok = wait(&p_full[x][pb], pu & 1);
            if (!ok) break;
            tc_fence_after();
            const uint32_t pcol = tbase + COL_S + pb * 128;
            for (int sc = 0; sc < NSUB; ++sc, ++vc) {
              const int slot = vc % VS;
              if (!wait(&v_full[slot], (vc / VS) & 1)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint64_t vd = vdesc0 + (uint64_t)(slot * (BOX >> 4));
#pragma unroll
              for (int x = 0; x < NWG; ++x)
#pragma unroll
                for (int kk = 0; kk < KW / 16; ++kk)
                  mma_bf16_ts(tbase + COL_O + sc * 64, pcol + x * KW + kk * 8,
                              vd + (uint64_t)((KW / 16 * x + kk) * 128), IDESC_O,
                              (kt == 0 && x == 0 && kk == 0) ? 0u : 1u);
              tc_commit(&v_empty[slot]);
            }
            if (!ok) break;
            tc_commit(&pv_done[pb]);
          }
          if (ok) tc_commit(&o_ready);
        }
      }
      if (!ok) abort_flag = 1;
    }
    __syncwarp();
  } else if (warp < W_EPI) {
    // ------------------------------------------------------------------ softmax, keys KW x .. of every tile
    const int x = warp >> 2;
    const int row = tid & 127;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const uint32_t col_o = tbase + lane_off + COL_O + x * DW;  // this warpgroup's head dims of O (rescale)
    int tile = 0, item = 0;
    bool quit = false;
    for (int n = 0, u; (u = cta_unit(sched, units, n)) >= 0 && !quit; ++n) {
      int b, h, qt;
      decode(u, b, h, qt);
      for (int pass = 0; pass < 2 && !quit; ++pass, ++item) {
        float m = -INFINITY, l = 0.f;
        for (int kt = 0; kt <= qt; ++kt, ++tile) {
          const int sb = tile % NSB;
          wait(&s_full[sb], (tile / NSB) & 1);
          tc_fence_after();
          __syncwarp();
          const uint32_t scol = tbase + lane_off + COL_S + sb * 128 + x * KW;
          uint32_t raw[KW];
#pragma unroll
          for (int c = 0; c < KW / 32; ++c) tmem_ld32_async(scol + 32 * c, raw + 32 * c);
          tmem_wait_ld();
          float v[KW];
#pragma unroll
          for (int i = 0; i < KW; ++i) v[i] = __uint_as_float(raw[i]);
          if (kt == qt) {  // the diagonal tile: keys past the query
#pragma unroll
            for (int i = 0; i < KW; ++i)
              if (x * KW + i > row) v[i] = -INFINITY;
          }
          float part[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) part[j] = v[j];
#pragma unroll
          for (int i = 8; i < KW; i += 16)
#pragma unroll
            for (int j = 0; j < 8; ++j) part[j] = max3(part[j], v[i + j], v[i + 8 + j]);
          const float tmax = max3(max3(part[0], part[1], part[2]), max3(part[3], part[4], part[5]),
                                  fmaxf(part[6], part[7])) * p.qscale;
          const bool saw_abort = abort_flag != 0;
          float mnew = m;
          bool slow = false;
          if (sync_or(1, SM_THREADS, tmax > m + kRescale || saw_abort)) {
            if (sync_or(1, SM_THREADS, saw_abort)) {
              quit = true;
              break;
            }
            ctl.tmax[x][row] = tmax;
            named_sync(2, SM_THREADS);
            float t2 = ctl.tmax[0][row];
#pragma unroll
            for (int y = 1; y < NWG; ++y) t2 = fmaxf(t2, ctl.tmax[y][row]);
            if (t2 > m + kRescale) mnew = t2;
            slow = true;
          }
          uint32_t w[KW / 2];
          uint64_t ls2[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) ls2[j] = 0ull;
          const uint64_t sc2 = f2_pack(p.qscale, p.qscale), nm2 = f2_pack(-mnew, -mnew);
#pragma unroll
          for (int i = 0; i < KW / 2; ++i) {
            float x0, x1;
            f2_unpack(f2_fma(f2_pack(v[2 * i], v[2 * i + 1]), sc2, nm2), x0, x1);
            const bool poly = i % kPolyEvery == kPolyEvery - 1;
            const float p0 = poly ? ex2_fma(x0) : ex2(x0);
            const float p1 = poly ? ex2_fma(x1) : ex2(x1);
            ls2[i & 3] = f2_add(ls2[i & 3], f2_pack(p0, p1));
            w[i] = pack_bf16x2(p0, p1);
          }
          float ls[8];
#pragma unroll
          for (int j = 0; j < 4; ++j) f2_unpack(ls2[j], ls[2 * j], ls[2 * j + 1]);
          if (slow) {
            const bool rescale = mnew != m && kt > 0;
            if (__any_sync(0xffffffffu, rescale)) {
              wait(&pv_done[(tile - 1) % NSB], ((tile - 1) / NSB) & 1);  // O holds every earlier tile of the pass
              tc_fence_after();
              __syncwarp();
              const float sc = rescale ? ex2(m - mnew) : 1.f;
#pragma unroll
              for (int c = 0; c < DW / 32; ++c) {
                float o[32];
                uint32_t ow[32];
                tmem_ld32(col_o + c * 32, o);
#pragma unroll
                for (int i = 0; i < 32; ++i) ow[i] = __float_as_uint(o[i] * sc);
                tmem_st32(col_o + c * 32, ow);
              }
              tmem_wait_st();
              l *= sc;
            }
            m = mnew;
          }
          l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
          tmem_st32(scol, w);
          tmem_wait_st();
          tc_fence_before();
          mbar_arrive(&p_full[x][sb]);
        }
        if (quit) break;
        if (item >= 1) wait(&l_free, (item - 1) & 1);
        ctl.lsum[x][row] = l;
        mbar_arrive(&l_full);
      }
    }
  } else if (warp < W_EPI + 4) {
    // ------------------------------------------------------------------ epilogue (thread = query row)
    const int row = tid & 127;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const bool q_loader = tid == W_EPI * 32;
    auto load_q = [&](int n, int u) {  // unit u (the CTA's n-th) into the query chunks, each once it is free
      int b, h, qt;
      decode(u, b, h, qt);
      for (int c = 0; c < DC; ++c) {
        if (n >= 1 && !wait(&q_empty[c], (n - 1) & 1)) return;
        mbar_arrive_expect_tx(&q_full[c], CHUNK);
        unsigned char* dst = smem + Q_OFF + c * CHUNK;
        tma_load_4d(dst, &qmap, c * 128, qt * BM, h, b, &q_full[c]);
        tma_load_4d(dst + BOX, &qmap, c * 128 + 64, qt * BM, h, b, &q_full[c]);
        issued_q = n * DC + c + 1;  // chunk loads issued
      }
    };
    if (q_loader) {
      prefetch_tmap(&qmap);
      const int u0 = cta_unit(sched, units, 0);
      if (u0 >= 0) load_q(0, u0);
    }
    int item = 0;
    for (int n = 0, u; (u = cta_unit(sched, units, n)) >= 0 && !abort_flag; ++n) {
      int b, h, qt;
      decode(u, b, h, qt);
      for (int pass = 0; pass < 2 && !abort_flag; ++pass, ++item) {
        if (pass == 1 && q_loader) {  // the next unit's queries, as the last S MMAs of this one free the chunks
          const int un = cta_unit(sched, units, n + 1);
          if (un >= 0) load_q(n + 1, un);
        }
        if (!wait(&o_ready, item & 1)) break;
        if (!wait(&l_full, item & 1)) break;
        tc_fence_after();
        __syncwarp();
        float l = 0.f;
#pragma unroll
        for (int y = 0; y < NWG; ++y) l += ctl.lsum[y][row];
        mbar_arrive(&l_free);
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const int q = qt * BM + row;
        __nv_bfloat16* dst =
            p.out + (int64_t)b * p.out_sb + (int64_t)q * p.out_sw + (int64_t)h * p.out_sh + pass * DH;
#pragma unroll 1
        for (int c = 0; c < DH / 64; ++c) {
          uint32_t r0[64];
          tmem_ld32_async(tbase + lane_off + COL_O + c * 64, r0);
          tmem_ld32_async(tbase + lane_off + COL_O + c * 64 + 32, r0 + 32);
          tmem_wait_ld();
          if (c == DH / 64 - 1) {  // O is in registers: the next pass may overwrite it
            tc_fence_before();
            mbar_arrive(&o_free);
          }
          if (q < p.width) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              uint32_t w4[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int k = 8 * i + 2 * j;
                w4[j] = pack_bf16x2(__uint_as_float(r0[k]) * inv, __uint_as_float(r0[k + 1]) * inv);
              }
              *reinterpret_cast<uint4*>(dst + c * 64 + i * 8) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
            }
          }
        }
      }
    }
  }
  __syncthreads();
  if (abort_flag) {
    if (tid == 0) raise_status(p.status, kStatusTimeout);
    if (tid == W_MMA * 32 || tid == W_MMA_PV * 32) {
      tc_commit(&drain);
      mbar_wait(&drain, 0);
    }
    if (tid == W_LOADK * 32) {
      for (int i = issued_k > KS ? issued_k - KS : 0; i < issued_k; ++i) mbar_wait(&k_full[i % KS], (i / KS) & 1);
      for (int i = issued_v > VS ? issued_v - VS : 0; i < issued_v; ++i) mbar_wait(&v_full[i % VS], (i / VS) & 1);
      // the latest load of every query chunk (load i fills chunk i % DC for the (i / DC)-th time)
      for (int i = issued_q > DC ? issued_q - DC : 0; i < issued_q; ++i) mbar_wait(&q_full[i % DC], (i / DC) & 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == W_EPI) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
}

bool make_map(CUtensorMap* map, const void* base, int64_t b, int64_t h, int64_t w, int64_t sb, int64_t sh,
              int64_t sw) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  if (!fn) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)b};
  cuuint64_t strides[3] = {(cuuint64_t)sw * 2, (cuuint64_t)sh * 2, (cuuint64_t)sb * 2};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace prefillw

cudaError_t launch_prefill_wide(const PrefillArgs& a, cudaStream_t stream) {
  using namespace prefillw;
  CUtensorMap qm, km, vm;
  if (!make_map(&qm, a.q, a.batch, a.heads, a.width, a.q_sb, a.q_sh, a.q_sw) ||
      !make_map(&km, a.k, a.batch, a.heads, a.width, a.k_sb, a.k_sh, a.k_sw) ||
      !make_map(&vm, a.v, a.batch, a.heads, a.width, a.v_sb, a.v_sh, a.v_sw))
    return cudaErrorInvalidValue;
  static bool configured = false;
  if (!configured) {
    cudaError_t e =
        cudaFuncSetAttribute(prefill_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  Params p;
  p.batch = a.batch;
  p.heads = a.heads;
  p.width = a.width;
  p.qtiles = (a.width + BM - 1) / BM;
  p.qscale = a.scale * kLog2e;
  p.group = omni::prefill_group(a.batch * a.heads);
  p.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  p.out_sb = a.o_sb;
  p.out_sw = a.o_sw;
  p.out_sh = a.o_sh;
  p.status = a.status;
  const int units = a.batch * a.heads * p.qtiles;
  int grid = device_sm_count();
  if (grid > units) grid = units;
  if (grid <= 0) return cudaSuccess;
  const Sched* sched = prefill_schedule(p.batch, p.heads, p.qtiles, p.group, grid);
  return launch_dependent(prefill_wide_kernel, dim3(grid), dim3(THREADS), (size_t)SMEM_BYTES, stream, qm, km, vm, p,
                          sched ? *sched : prefill_round_robin());
}

}  // namespace omni
