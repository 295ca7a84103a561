// Causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), bf16, head_dim 128.
//
// out[b, w, h] = softmax(q[b, h, w] . k[b, h, :w+1]^T * scale) . v[b, h, :w+1]   for w < W
// (F.scaled_dot_product_attention(q, k, v, is_causal=True) of the reference's prefill, decode.py:171; the
// reference-semantics form is modeling.py:398-399). Right-padded rows need nothing special: a valid query never
// sees a later (pad) key.
//
// Work unit: (row b, head h, 128-query tile qt) over key tiles 0..qt; units are taken by a persistent grid of one
// CTA per SM in groups of (b, h) pairs, heaviest first within a group (unit_of). Roles (512 threads):
//   warp 12 TMA: the K tiles (3-slot ring, two 64-column boxes each, 128-byte swizzle); warp 14 TMA: the V tiles;
//           the query tiles (2 slots) are loaded two units ahead by the first epilogue thread
//   warp 13 MMA: S = Q K^T into TMEM (M=128 queries, N=128 keys), triple-buffered, so that S(t + 3) needs only
//           O += P(t) V to have completed and the scores are ready before the softmax asks for them;
//   warp 15 MMA: O += P V with P read from TMEM (the tcgen05 "A in TMEM" form). Two issuing threads, because one
//           thread issues a tcgen05.mma in about 55 clocks at best (measured), while a 128x128x16 MMA takes the
//           tensor core about 64: a single issuer with its waits left the tensor core idle half the time.
//   warps 0-3 / 4-7  softmax warpgroups x = 0 / 1: thread t of warpgroup x owns query row t and the keys 64x .. 64x+63
//           of every tile, so twice the softmax warps per SM each form half a tile's exponentials. The two keep one
//           running max per row: each tile one barrier over both warpgroups asks whether any row's scores pass its
//           max by 2^8 (log2 units); only then are the tile maxima exchanged, the max raised and O rescaled in TMEM
//           (each warpgroup its 64 head dims). P (bf16 pairs) is written over the warpgroup's half of S in TMEM.
//           The scale-and-subtract and the row sums use the packed f32x2 FMA / add (two elements per instruction),
//           and one probability pair in four is exponentiated on the FMA pipe (ex2_fma) instead of the
//           special-function unit, which the exponentials otherwise saturate.
//   warps 8-11 epilogue: O / (l_0 + l_1) of each unit as bf16 rows, while the softmax warpgroups go on with the next.
// TMEM: S0 [0,128) S1 [128,256) S2 [256,384) O [384,512); P of S buffer j, half x at 128j + 64x .. +32.

#include <cudaTypedefs.h>
#include <math.h>

#include <array>
#include <map>
#include <memory>
#include <mutex>
#include <queue>
#include <vector>

#include "attention.cuh"
#include "prefill.cuh"
#include "prefill_common.cuh"
#include "tc.cuh"
#include "trace.cuh"

namespace omni {
namespace prefill {

using namespace pfx;

constexpr int D = 128;
constexpr int BM = 128;  // queries per tile
constexpr int BN = 128;  // keys per tile
constexpr int TILE = BN * D * 2;
constexpr int BOX = BN * 64 * 2;
constexpr int QS = 2, KS = 3, VS = 2;  // query tiles (two units), K and V rings, in shared memory
constexpr int Q_OFF = 0;
constexpr int K_OFF = Q_OFF + QS * TILE;
constexpr int V_OFF = K_OFF + KS * TILE;
constexpr int SMEM_BYTES = V_OFF + VS * TILE;
constexpr int NSB = 3;  // S buffers in TMEM: S(t + 3) needs only O += P(t) V to have completed
constexpr int NWG = 2;        // softmax warpgroups; warpgroup x owns keys KW x .. KW x + KW - 1 of every tile
constexpr int KW = BN / NWG;  // keys per softmax warpgroup (a multiple of the 16-key MMA step)
constexpr int DW = D / NWG;   // head dims of O each softmax warpgroup rescales
constexpr int W_EPI = 4 * NWG, W_LOADK = W_EPI + 4, W_MMA = W_LOADK + 1, W_LOADV = W_LOADK + 2, W_MMA_PV = W_LOADK + 3;
constexpr int THREADS = 32 * (W_MMA_PV + 1);  // softmax, Q loader + epilogue, K loads, S MMAs, V loads, PV MMAs
constexpr int SM_THREADS = 128 * NWG;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S = 0, COL_O = 384;  // S buffer j at 128 j
constexpr uint32_t IDESC_S = idesc_bf16(BM, BN, 0, 0);
constexpr uint32_t IDESC_O = idesc_bf16(BM, D, 0, 1);
constexpr float kRescale = 8.f;
#ifndef OMNI_PREFILL_POLY_EVERY
#define OMNI_PREFILL_POLY_EVERY 4
#endif
constexpr int kPolyEvery = OMNI_PREFILL_POLY_EVERY;  // probabilities of one pair in this many by ex2_fma

struct Params {
  int batch, heads, width, qtiles;
  int group;  // (row, head) pairs per scheduling group
  float qscale;  // scale * log2(e)
  const __nv_bfloat16* q;
  int64_t q_sb, q_sh, q_sw;  // q[b, h, w, :] strides (elements)
  __nv_bfloat16* out;
  int64_t out_sb, out_sw, out_sh;  // out[b, w, h, :] strides (elements)
  int* status;
};

OMNI_DEV void unit_of(const Params& p, int u, int& b, int& h, int& qt) {
  pfx::unit_of(p.batch, p.heads, p.qtiles, p.group, u, b, h, qt);
}

// The CTA's control block: barriers, the row maxima exchanged between the softmax warpgroups, the unit's row sums
// for the epilogue, flags. One static struct, padded to 1024 bytes, so that the dynamic tile ring after it starts
// 1024-aligned (the kernel checks, and reports status bit 4 otherwise).
struct alignas(1024) Ctl {
  uint64_t k_full[KS], k_empty[KS], v_full[VS], v_empty[VS], q_full[QS], q_empty[QS];
  uint64_t s_full[NSB], p_full[NWG][NSB], pv_done[NSB], o_ready, o_free, l_full, l_free, drain;
  float tmax[NWG][BM];  // [warpgroup][row]: a tile's scaled row maxima, on the rare tiles that raise a max
  float lsum[NWG][BM];  // [warpgroup][row]: the unit's row sums for the epilogue
  uint32_t tmem_base;
  int abort_flag, issued_k, issued_v, issued_q;  // loads the producers issued
};
static_assert(sizeof(Ctl) + SMEM_BYTES <= 232448, "shared memory per block");
static_assert(NSB * 128 + D <= TMEM_COLS, "S buffers and O in TMEM");

__global__ void __launch_bounds__(THREADS, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
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
  if (smem_addr(smem) & 1023u) {  // the swizzled tiles need a 1024-aligned ring
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
    for (int j = 0; j < QS; ++j) {
      mbar_init(&q_full[j], 1);
      mbar_init(&q_empty[j], 1);
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
  if (tid == 0) OMNI_TRACE_AT(1599);
  OMNI_TRACE_CTA(0);
  const uint32_t tbase = ctl.tmem_base;
  // Every wait gives up at once when another role has given up (abort_flag), else after the bounded time.
  auto wait = [&](uint64_t* bar, uint32_t parity) -> bool {
    if (mbar_wait_or(bar, parity, &abort_flag)) return true;
    abort_flag = 1;
    return false;
  };

  if (warp == W_LOADK || warp == W_LOADV) {
    // ------------------------------------------------------------------ producers
    if (lane == 0) {
      const bool is_k = warp == W_LOADK;
      const CUtensorMap* map = is_k ? &kmap : &vmap;
      prefetch_tmap(map);
      const int ns = is_k ? KS : VS;
      unsigned char* ring = smem + (is_k ? K_OFF : V_OFF);
      uint64_t* full = is_k ? k_full : v_full;
      uint64_t* empty = is_k ? k_empty : v_empty;
      int tile = 0;
      for (int n = 0, u; (u = cta_unit(sched, units, n)) >= 0 && !abort_flag; ++n) {
        int b, h, qt;
        unit_of(p, u, b, h, qt);
        for (int kt = 0; kt <= qt && !abort_flag; ++kt, ++tile) {
          const int slot = tile % ns, use = tile / ns;
          if (use >= 1 && !wait(&empty[slot], (use - 1) & 1)) break;
          mbar_arrive_expect_tx(&full[slot], TILE);
          tma_load_4d(ring + slot * TILE, map, 0, kt * BN, h, b, &full[slot]);
          tma_load_4d(ring + slot * TILE + BOX, map, 64, kt * BN, h, b, &full[slot]);
          if (is_k) issued_k = tile + 1;
          else issued_v = tile + 1;
          OMNI_TRACE_AT(tile * 8 + (is_k ? 0 : 1));
        }
      }
    }
    __syncwarp();
  } else if (warp == W_MMA) {
    // ------------------------------------------------------------------ S issuer: S[t % NSB] = Q K(t)^T
    // S[t % NSB] is free once O += P(t - NSB) V has completed (P(t - NSB) lies over it); the unit's Q slot is
    // released after its last S (q_empty).
    if (lane == 0) {
      // Slot s's descriptor is slot 0's with the start address (in 16-byte units, 14 bits) moved on by s tiles.
      const uint64_t kdesc0 = smem_desc(smem_addr(smem + K_OFF), 16, 1024, kLayoutSw128);
      const uint64_t qdesc0 = smem_desc(smem_addr(smem + Q_OFF), 16, 1024, kLayoutSw128);
      int tile = 0, nunit = 0, sb = 0;
      bool ok = true;
      for (int u; (u = cta_unit(sched, units, nunit)) >= 0 && ok && !abort_flag; ++nunit) {
        int b, h, qt;
        unit_of(p, u, b, h, qt);
        const int qslot = nunit % QS;
        if (!wait(&q_full[qslot], (nunit / QS) & 1)) break;
        const uint64_t qd = qdesc0 + (uint64_t)(qslot * (TILE >> 4));
        for (int kt = 0; kt <= qt; ++kt, ++tile, sb = sb == NSB - 1 ? 0 : sb + 1) {
          const int slot = tile % KS;
          if (tile >= NSB && !wait(&pv_done[sb], ((tile - NSB) / NSB) & 1)) {
            ok = false;
            break;
          }
          if (!wait(&k_full[slot], (tile / KS) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t dcol = tbase + COL_S + sb * 128;
          const uint64_t kd = kdesc0 + (uint64_t)(slot * (TILE >> 4));
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t off = (uint64_t)((((kk >> 2) * BOX + (kk & 3) * 32) >> 4));
            mma_bf16_ss(dcol, qd + off, kd + off, IDESC_S, kk > 0 ? 1u : 0u);
          }
          tc_commit(&s_full[sb]);
          tc_commit(&k_empty[slot]);
          if (kt == qt) tc_commit(&q_empty[qslot]);  // the unit's last read of its query tile
          OMNI_TRACE_AT(tile * 8 + 2);
        }
      }
    }
    __syncwarp();
  } else if (warp == W_MMA_PV) {
    // ------------------------------------------------------------------ PV issuer: O += P(t) V(t)
    // The two key halves in turn, as their softmax warpgroups finish; a unit's first tile overwrites O once the
    // epilogue has read the previous unit's (o_free).
    if (lane == 0) {
      const uint64_t vdesc0 = smem_desc(smem_addr(smem + V_OFF), BOX, 1024, kLayoutSw128);
      int tile = 0, nunit = 0;
      bool ok = true;
      for (int u; (u = cta_unit(sched, units, nunit)) >= 0 && ok && !abort_flag; ++nunit) {
        int b, h, qt;
        unit_of(p, u, b, h, qt);
        for (int kt = 0; kt <= qt; ++kt, ++tile) {
          const int pb = tile % NSB, pu = tile / NSB;
          const int slot = tile % VS;
          if (kt == 0 && nunit >= 1 && !wait(&o_free, (nunit - 1) & 1)) {
            ok = false;
            break;
          }
          if (!wait(&v_full[slot], (tile / VS) & 1)) {
            ok = false;
            break;
          }
          const uint64_t vd = vdesc0 + (uint64_t)(slot * (TILE >> 4));
          const uint32_t pcol = tbase + COL_S + pb * 128;
#pragma unroll
          for (int x = 0; x < NWG; ++x) {
            if (!wait(&p_full[x][pb], pu & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < KW / 16; ++kk)
              mma_bf16_ts(tbase + COL_O, pcol + x * KW + kk * 8, vd + (uint64_t)((KW / 16 * x + kk) * 128), IDESC_O,
                          (kt == 0 && x == 0 && kk == 0) ? 0u : 1u);
          }
          if (!ok) break;
          tc_commit(&pv_done[pb]);
          tc_commit(&v_empty[slot]);
          OMNI_TRACE_AT(tile * 8 + 3);
        }
        if (ok) tc_commit(&o_ready);
      }
    }
    __syncwarp();
  } else if (warp < W_EPI) {
    // ------------------------------------------------------------------ softmax, keys KW x .. of every tile
    // The warpgroups leave their loops only on a decision taken at a barrier over all their threads, so that no
    // thread waits at a barrier the others have left: a wait that gives up sets abort_flag and the thread goes on
    // to the tile's barrier, where every thread sees it.
    const int x = warp >> 2;
    const int row = tid & 127;  // query row within the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const uint32_t col_o = tbase + lane_off + COL_O + x * DW;  // this warpgroup's head dims of O (rescale)
    int tile = 0, nunit = 0;
    bool quit = false;
    for (int u; (u = cta_unit(sched, units, nunit)) >= 0 && !quit; ++nunit) {
      int b, h, qt;
      unit_of(p, u, b, h, qt);
      float m = -INFINITY, l = 0.f;
      for (int kt = 0; kt <= qt; ++kt, ++tile) {
        const int sb = tile % NSB;
        if (row == 0 && x == 0 && tile < 300) OMNI_TRACE_AT(2400 + 1200 + tile);
        wait(&s_full[sb], (tile / NSB) & 1);
        if (row == 0 && x < 2) OMNI_TRACE_AT(tile * 8 + 4 + 2 * x);
        tc_fence_after();
        __syncwarp();
        const uint32_t scol = tbase + lane_off + COL_S + sb * 128 + x * KW;
        uint32_t raw[KW];
#pragma unroll
        for (int c = 0; c < KW / 32; ++c) tmem_ld32_async(scol + 32 * c, raw + 32 * c);
        tmem_wait_ld();
        if (row == 0 && x == 0 && tile < 400) OMNI_TRACE_AT(2400 + tile * 4);
        float v[KW];
#pragma unroll
        for (int i = 0; i < KW; ++i) v[i] = __uint_as_float(raw[i]);
        if (kt == qt) {  // the diagonal tile: keys past the query
#pragma unroll
          for (int i = 0; i < KW; ++i)
            if (x * KW + i > row) v[i] = -INFINITY;
        }
        static_assert(KW % 16 == 0, "row max in 8 partials of two values per step");
        float part[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) part[j] = v[j];
#pragma unroll
        for (int i = 8; i < KW; i += 16)
#pragma unroll
          for (int j = 0; j < 8; ++j) part[j] = max3(part[j], v[i + j], v[i + 8 + j]);
        const float tmax = max3(max3(part[0], part[1], part[2]), max3(part[3], part[4], part[5]),
                                fmaxf(part[6], part[7])) * p.qscale;
        // One barrier per tile over the warpgroups: does any row need a higher max, or has any thread seen an abort?
        const bool saw_abort = abort_flag != 0;
        float mnew = m;
        bool slow = false;
        const bool any_raise = sync_or(1, SM_THREADS, tmax > m + kRescale || saw_abort);
        if (row == 0 && x == 0 && tile < 400) OMNI_TRACE_AT(2401 + tile * 4);
        if (any_raise) {
          if (sync_or(1, SM_THREADS, saw_abort)) {
            quit = true;
            break;
          }
          ctl.tmax[x][row] = tmax;
          named_sync(2, SM_THREADS);
          float t2 = ctl.tmax[0][row];  // the same in every warpgroup
#pragma unroll
          for (int y = 1; y < NWG; ++y) t2 = fmaxf(t2, ctl.tmax[y][row]);
          if (t2 > m + kRescale) mnew = t2;
          slow = true;
        }
        // Probabilities (bf16 pairs) over this warpgroup's keys, and the row sum; formed before any rescale of O, so
        // that the scores are dead by then (register pressure).
        uint32_t w[KW / 2];
        uint64_t ls2[4];  // row-sum partials, two per packed register
#pragma unroll
        for (int j = 0; j < 4; ++j) ls2[j] = 0ull;
        const uint64_t sc2 = f2_pack(p.qscale, p.qscale), nm2 = f2_pack(-mnew, -mnew);
#pragma unroll
        for (int i = 0; i < KW / 2; ++i) {
          // x = s * scale - max for a pair in one packed FMA; one pair in kPolyEvery exponentiated on the FMA pipe,
          // the rest on the special-function unit.
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
            wait(&pv_done[(tile - 1) % NSB], ((tile - 1) / NSB) & 1);  // O holds every earlier tile
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
        if (row == 0 && x == 0 && tile < 400) OMNI_TRACE_AT(2402 + tile * 4);
        // P over this warpgroup's scores, which are in registers already.
        if constexpr (KW / 2 == 32) tmem_st32(scol, w);
        else tmem_st16(scol, w);
        tmem_wait_st();
        if (row == 0 && x == 0 && tile < 400) OMNI_TRACE_AT(2403 + tile * 4);
        tc_fence_before();
        mbar_arrive(&p_full[x][sb]);
        if (row == 0 && x < 2) OMNI_TRACE_AT(tile * 8 + 5 + 2 * x);
      }
      if (quit) break;
      // The unit's row sums of these keys for the epilogue, once it has read the previous unit's (a unit of one or
      // two tiles can be finished before that, and l_full must not complete two phases ahead of its waiter).
      if (nunit >= 1) wait(&l_free, (nunit - 1) & 1);
      ctl.lsum[x][row] = l;
      mbar_arrive(&l_full);
    }
  } else if (warp < W_EPI + 4) {
    // ------------------------------------------------------------------ epilogue (thread = query row)
    const int row = tid & 127;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    // One thread also loads the query tiles, two units ahead: unit n + 2's goes into unit n's slot once unit n's last
    // S has completed (q_empty, before its O is ready), so a unit's first S never waits for its queries.
    const bool q_loader = tid == W_EPI * 32;
    auto load_q = [&](int n, int u) {
      int b, h, qt;
      unit_of(p, u, b, h, qt);
      const int qslot = n % QS;
      mbar_arrive_expect_tx(&q_full[qslot], TILE);
      tma_load_4d(smem + Q_OFF + qslot * TILE, &qmap, 0, qt * BM, h, b, &q_full[qslot]);
      tma_load_4d(smem + Q_OFF + qslot * TILE + BOX, &qmap, 64, qt * BM, h, b, &q_full[qslot]);
      issued_q = n + 1;
    };
    if (q_loader) {
      prefetch_tmap(&qmap);
      for (int n = 0, u; n < QS && (u = cta_unit(sched, units, n)) >= 0; ++n) load_q(n, u);
    }
    int nunit = 0;
    for (int u; (u = cta_unit(sched, units, nunit)) >= 0 && !abort_flag; ++nunit) {
      int b, h, qt;
      unit_of(p, u, b, h, qt);
      const int ahead = q_loader ? cta_unit(sched, units, nunit + QS) : -1;
      if (ahead >= 0) {
        if (!wait(&q_empty[nunit % QS], (nunit / QS) & 1)) break;
        load_q(nunit + QS, ahead);
      }
      if (!wait(&o_ready, nunit & 1)) break;
      if (!wait(&l_full, nunit & 1)) break;
      if (row == 0) OMNI_TRACE_AT(1600 + nunit * 2);
      tc_fence_after();
      __syncwarp();
      float l = 0.f;
#pragma unroll
      for (int y = 0; y < NWG; ++y) l += ctl.lsum[y][row];
      mbar_arrive(&l_free);
      const float inv = l > 0.f ? 1.f / l : 0.f;
      const int q = qt * BM + row;
      __nv_bfloat16* dst = p.out + (int64_t)b * p.out_sb + (int64_t)q * p.out_sw + (int64_t)h * p.out_sh;
      // O in two halves of 64 columns (two loads in flight per wait), released to the next unit's first P V once the
      // second half is in registers, before it is scaled and stored (measured: 183.0 us per config-4 call against
      // 186.5 us with four 32-column reads and the release after the last store).
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t r0[64];
        tmem_ld32_async(tbase + lane_off + COL_O + c * 64, r0);
        tmem_ld32_async(tbase + lane_off + COL_O + c * 64 + 32, r0 + 32);
        tmem_wait_ld();
        if (c == 1) {
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
      if (row == 0) OMNI_TRACE_AT(1601 + nunit * 2);
    }
  }
  __syncthreads();
  if (abort_flag) {
    if (tid == 0) raise_status(p.status, kStatusTimeout);
    if (tid == W_MMA * 32 || tid == W_MMA_PV * 32) {
      // Every MMA an issuer thread issued has completed once its commit arrives (two issuers: two arrivals).
      tc_commit(&drain);
      mbar_wait(&drain, 0);
    }
    if (tid == W_LOADK * 32) {
      // Let the latest load of every slot land (a slot is refilled only after its previous load was consumed).
      for (int i = issued_k > KS ? issued_k - KS : 0; i < issued_k; ++i) mbar_wait(&k_full[i % KS], (i / KS) & 1);
      for (int i = issued_v > VS ? issued_v - VS : 0; i < issued_v; ++i) mbar_wait(&v_full[i % VS], (i / VS) & 1);
      for (int i = issued_q > QS ? issued_q - QS : 0; i < issued_q; ++i) mbar_wait(&q_full[i % QS], (i / QS) & 1);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == W_EPI) {
    tc_fence_after();
    tmem_dealloc(tbase, TMEM_COLS);
  }
  OMNI_TRACE_CTA(1);
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

}  // namespace prefill

// (row, head) pairs per scheduling group: about 16, so that one group's units cover the grid once or twice and its
// K/V (under 13 MB at width 1500) stay in L2 while the grid works through them. OMNIASR_PREFILL_GROUP overrides.
int prefill_group(int bh_count) {
  static const int env = [] {
    const char* e = getenv("OMNIASR_PREFILL_GROUP");
    return e ? atoi(e) : 0;
  }();
  int g = env > 0 ? env : 16;
  return g < bh_count ? g : bh_count;
}

// Fixed cost of a unit in key tiles (measured: a unit's first tile takes about 1.6 tiles' time).
constexpr float kPrefillUnitCost = 0.6f;

// The list schedule of `units` units (unit_of's numbering) over `grid` CTAs, cached per shape.
const pfx::Sched* prefill_schedule(int batch, int heads, int qtiles, int group, int grid) {
  static const bool off = [] {  // OMNIASR_PREFILL_SCHED=0: round-robin (for comparisons)
    const char* e = getenv("OMNIASR_PREFILL_SCHED");
    return e && atoi(e) == 0;
  }();
  const int units = batch * heads * qtiles;
  if (off || units > pfx::kSchedUnits || grid > pfx::kSchedCtas) return nullptr;
  static std::mutex mu;
  static std::map<std::array<int, 5>, std::unique_ptr<pfx::Sched>> cache;
  const std::array<int, 5> key{batch, heads, qtiles, group, grid};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second.get();
  auto s = std::make_unique<pfx::Sched>();
  std::vector<std::vector<uint16_t>> lists(grid);
  using Slot = std::pair<float, int>;  // (time the CTA is free, CTA)
  std::priority_queue<Slot, std::vector<Slot>, std::greater<Slot>> free_at;
  for (int c = 0; c < grid; ++c) free_at.push({0.f, c});
  const int bh_count = batch * heads;
  for (int u = 0; u < units; ++u) {
    const int per_group = group * qtiles;  // unit_of's numbering, on the host
    const int g0 = (u / per_group) * group;
    const int gsize = std::min(group, bh_count - g0);
    const int qt = qtiles - 1 - (u - g0 * qtiles) / gsize;
    const Slot c = free_at.top();
    free_at.pop();
    lists[c.second].push_back((uint16_t)u);
    free_at.push({c.first + (float)(qt + 1) + kPrefillUnitCost, c.second});
  }
  s->on = 1;
  int k = 0;
  for (int c = 0; c < grid; ++c) {
    s->start[c] = (uint16_t)k;
    for (uint16_t u : lists[c]) s->unit[k++] = u;
  }
  s->start[grid] = (uint16_t)k;
  return cache.emplace(key, std::move(s)).first->second.get();
}

const pfx::Sched& prefill_round_robin() {
  static const pfx::Sched r = [] {
    pfx::Sched x{};
    x.on = 0;
    return x;
  }();
  return r;
}

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t stream) {
  using namespace prefill;
  CUtensorMap qm, km, vm;
  if (!make_map(&qm, a.q, a.batch, a.heads, a.width, a.q_sb, a.q_sh, a.q_sw) ||
      !make_map(&km, a.k, a.batch, a.heads, a.width, a.k_sb, a.k_sh, a.k_sw) ||
      !make_map(&vm, a.v, a.batch, a.heads, a.width, a.v_sb, a.v_sh, a.v_sw))
    return cudaErrorInvalidValue;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
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
  p.q = reinterpret_cast<const __nv_bfloat16*>(a.q);
  p.q_sb = a.q_sb;
  p.q_sh = a.q_sh;
  p.q_sw = a.q_sw;
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
  return launch_dependent(prefill_kernel, dim3(grid), dim3(THREADS), (size_t)SMEM_BYTES, stream, qm, km, vm, p,
                          sched ? *sched : prefill_round_robin());
}

}  // namespace omni
