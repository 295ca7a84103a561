// Causal prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), bf16, head_dim 128.
//
// out[b, w, h] = softmax(q[b, h, w] . k[b, h, :w+1]^T * scale) . v[b, h, :w+1]   for w < W
// (F.scaled_dot_product_attention(q, k, v, is_causal=True) of the reference's prefill, decode.py:171; the
// reference-semantics form is modeling.py:398-399). Right-padded rows need nothing special: a valid query never
// sees a later (pad) key.
//
// Work unit: (row b, head h, 128-query tile qt) over key tiles 0..qt; units are taken by a persistent grid of one
// CTA per SM in groups of (b, h) pairs, heaviest first within a group (unit_of). Roles (480 threads):
//   warp 12 TMA: the query tiles (2 slots; two 64-column boxes, 128-byte swizzle) and the K tiles (3-slot ring)
//   warp 14 TMA: the V tiles (2-slot ring)
//   warp 13 MMA: S = Q K^T into TMEM (M=128 queries, N=128 keys, double-buffered); then, for each half x of the
//           tile's keys, O_x += P_x V_x with P_x read from TMEM (the tcgen05 "A in TMEM" form, K = 64 keys)
//   warps 0-3 / 4-7  softmax warpgroups x = 0 / 1: thread t of warpgroup x owns query row t and the keys
//           64x .. 64x+63 of every tile. Each keeps its own running max and sum over its half of the keys and its
//           own accumulator O_x, so the two never synchronise: twice the softmax warps per SM, each with half a
//           tile's exponentials, on independent chains. The running max is raised only when a row's scores pass it
//           by 2^8, and only then is the row's O_x rescaled in TMEM. P_x (bf16 pairs) is written over the
//           warpgroup's own half of S in TMEM.
//   warps 8-11 epilogue: per unit, O = (O_0 2^(m_0 - M) + O_1 2^(m_1 - M)) / (l_0 2^(m_0 - M) + l_1 2^(m_1 - M)),
//           M = max(m_0, m_1), written as bf16 rows, while the softmax warpgroups start the next unit.
// TMEM: S0 [0,128) S1 [128,256) O_0 [256,384) O_1 [384,512); P_x of buffer j at columns 128j + 64x .. +32.

#include <cudaTypedefs.h>
#include <math.h>

#include "attention.cuh"
#include "prefill.cuh"
#include "tc.cuh"
#include "trace.cuh"

namespace omni {
namespace prefill {

constexpr int D = 128;
constexpr int BM = 128;  // queries per tile
constexpr int BN = 128;  // keys per tile
constexpr int TILE = BN * D * 2;
constexpr int BOX = BN * 64 * 2;
constexpr int QS = 2, KS = 3, VS = 2;
constexpr int Q_OFF = 0;
constexpr int K_OFF = Q_OFF + QS * TILE;
constexpr int V_OFF = K_OFF + KS * TILE;
// The tile ring fills the dynamic shared memory exactly: with the 3 KB control block (one static, 1024-aligned
// struct) the CTA uses 227 KB, the per-block maximum, so there is no room for alignment slack; the kernel checks
// that the dynamic region starts 1024-aligned (as the 128-byte swizzle needs) and reports status bit 4 otherwise.
constexpr int SMEM_BYTES = V_OFF + VS * TILE;
constexpr int THREADS = 480;  // warps 0-7 softmax, 8-11 epilogue, 12 K/Q loads, 13 MMA, 14 V loads
constexpr int W_EPI = 8, W_LOADK = 12, W_MMA = 13, W_LOADV = 14;
constexpr uint32_t TMEM_COLS = 512;
constexpr uint32_t COL_S = 0, COL_O = 256;  // S buffer j at 128 j; O_x at 256 + 128 x
constexpr uint32_t IDESC_S = idesc_bf16(BM, BN, 0, 0);
constexpr uint32_t IDESC_O = idesc_bf16(BM, D, 0, 1);
constexpr float kRescale = 8.f;

struct Params {
  int batch, heads, width, qtiles;
  int group;  // (row, head) pairs per scheduling group
  float qscale;  // scale * log2(e)
  __nv_bfloat16* out;
  int64_t out_sb, out_sw, out_sh;  // out[b, w, h, :] strides (elements)
  int* status;
};

// D (TMEM) = A (TMEM) x B (smem) [+ D]; issued by one thread.
OMNI_DEV void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

OMNI_DEV void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 columns of this thread's lane without waiting (complete after tmem_wait_ld()).
OMNI_DEV void tmem_ld32_async(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Two floats rounded to bf16 and packed (lo in the low half).
OMNI_DEV uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

OMNI_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

OMNI_DEV void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

OMNI_DEV void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

OMNI_DEV void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Unit u -> (b, h, qt). The (row, head) pairs are taken in groups of p.group, and a group's units heaviest query
// tile first: the CTAs running at one time then read the K/V of about one group, which stays in L2.
OMNI_DEV void unit_of(const Params& p, int u, int& b, int& h, int& qt) {
  const int bh_count = p.batch * p.heads;
  const int per_group = p.group * p.qtiles;
  const int g0 = (u / per_group) * p.group;
  const int gsize = min(p.group, bh_count - g0);
  const int r = u - g0 * p.qtiles;
  qt = p.qtiles - 1 - r / gsize;
  const int bh = g0 + r % gsize;
  b = bh / p.heads;
  h = bh % p.heads;
}

// The CTA's control block: barriers, the unit's per-row (max, sum) of each half for the epilogue, flags. One static
// struct, padded to a multiple of 1024 bytes, so that the dynamic tile ring after it starts 1024-aligned.
struct alignas(1024) Ctl {
  uint64_t q_full[QS], q_empty[QS], k_full[KS], k_empty[KS], v_full[VS], v_empty[VS];
  uint64_t s_full[2], p_full[2][2], pv_done[2][2], o_ready, o_free, ml_full, ml_free, drain;
  float2 ml[2][BM];  // [half x][row]
  uint32_t tmem_base;
  int abort_flag, issued_k, issued_v, issued_q;  // loads the producers issued
};
static_assert(sizeof(Ctl) == 3072, "control block + tile ring = the 227 KB per-block maximum");
static_assert(sizeof(Ctl) + SMEM_BYTES <= 232448, "shared memory per block");

__global__ void __launch_bounds__(THREADS, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const Params p) {
  extern __shared__ __align__(1024) unsigned char smem[];
  __shared__ Ctl ctl;
  uint64_t *q_full = ctl.q_full, *q_empty = ctl.q_empty, *k_full = ctl.k_full, *k_empty = ctl.k_empty;
  uint64_t *v_full = ctl.v_full, *v_empty = ctl.v_empty, *s_full = ctl.s_full;
  uint64_t(*p_full)[2] = ctl.p_full;
  uint64_t(*pv_done)[2] = ctl.pv_done;
  uint64_t &o_ready = ctl.o_ready, &o_free = ctl.o_free, &ml_full = ctl.ml_full, &ml_free = ctl.ml_free;
  uint64_t& drain = ctl.drain;
  float2(*ml_stash)[BM] = ctl.ml;
  uint32_t& tmem_base = ctl.tmem_base;
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
    for (int s = 0; s < QS; ++s) {
      mbar_init(&q_full[s], 1);
      mbar_init(&q_empty[s], 1);
    }
    for (int s = 0; s < KS; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    for (int x = 0; x < 2; ++x)
      for (int j = 0; j < 2; ++j) {
        mbar_init(&p_full[x][j], 128);
        mbar_init(&pv_done[x][j], 1);
      }
    mbar_init(&o_ready, 1);
    mbar_init(&o_free, 128);
    mbar_init(&ml_full, 256);
    mbar_init(&ml_free, 128);
    mbar_init(&drain, 1);
    mbar_fence_init();
    abort_flag = 0;
    issued_k = issued_v = issued_q = 0;
  }
  if (warp == W_EPI) tmem_alloc(&tmem_base, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  grid_dependency_wait();  // q, k, v may come from the kernel before (launched as a programmatic dependent)
  const uint32_t tbase = tmem_base;
  unsigned char* qs = smem + Q_OFF;
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
      prefetch_tmap(is_k ? &kmap : &vmap);
      if (is_k) prefetch_tmap(&qmap);
      int tile = 0, nunit = 0;
      for (int u = blockIdx.x; u < units && !abort_flag; u += gridDim.x, ++nunit) {
        int b, h, qt;
        unit_of(p, u, b, h, qt);
        if (is_k) {
          const int qslot = nunit % QS, quse = nunit / QS;
          if (quse >= 1 && !wait(&q_empty[qslot], (quse - 1) & 1)) break;
          mbar_arrive_expect_tx(&q_full[qslot], TILE);
          tma_load_4d(qs + qslot * TILE, &qmap, 0, qt * BM, h, b, &q_full[qslot]);
          tma_load_4d(qs + qslot * TILE + BOX, &qmap, 64, qt * BM, h, b, &q_full[qslot]);
          issued_q = nunit + 1;
        }
        for (int kt = 0; kt <= qt && !abort_flag; ++kt, ++tile) {
          const int ns = is_k ? KS : VS;
          const int slot = tile % ns, use = tile / ns;
          uint64_t* empty = is_k ? &k_empty[slot] : &v_empty[slot];
          uint64_t* full = is_k ? &k_full[slot] : &v_full[slot];
          if (use >= 1 && !wait(empty, (use - 1) & 1)) break;
          unsigned char* dst = smem + (is_k ? K_OFF : V_OFF) + slot * TILE;
          mbar_arrive_expect_tx(full, TILE);
          tma_load_4d(dst, is_k ? &kmap : &vmap, 0, kt * BN, h, b, full);
          tma_load_4d(dst + BOX, is_k ? &kmap : &vmap, 64, kt * BN, h, b, full);
          if (is_k) issued_k = tile + 1;
          else issued_v = tile + 1;
        }
      }
    }
    __syncwarp();
  } else if (warp == W_MMA) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int tile = 0, nunit = 0, qslot = 0;
      bool ok = true;
      auto scores = [&](int t) -> bool {  // S[t & 1] = Q K(t)^T (S[t & 1] was last read by O += P(t - 2) V)
        const int slot = t % KS;
        if (!wait(&k_full[slot], (t / KS) & 1)) return false;
        tc_fence_after();
        const uint32_t qa = smem_addr(qs + qslot * TILE), ka = smem_addr(smem + K_OFF + slot * TILE);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint64_t a = smem_desc(qa + (kk >> 2) * BOX + (kk & 3) * 32, 16, 1024, kLayoutSw128);
          const uint64_t bd = smem_desc(ka + (kk >> 2) * BOX + (kk & 3) * 32, 16, 1024, kLayoutSw128);
          mma_bf16_ss(tbase + COL_S + (t & 1) * 128, a, bd, IDESC_S, kk > 0 ? 1u : 0u);
        }
        tc_commit(&s_full[t & 1]);
        tc_commit(&k_empty[slot]);
        return true;
      };
      auto values = [&](int t, bool first_of_unit) -> bool {  // O_x += P_x(t) V_x(t), x = 0, 1
        const int pb = t & 1, pu = t >> 1;
        const int slot = t % VS;
        if (first_of_unit && nunit >= 1 && !wait(&o_free, (nunit - 1) & 1)) return false;
        if (!wait(&v_full[slot], (t / VS) & 1)) return false;
        const uint32_t va = smem_addr(smem + V_OFF + slot * TILE);
#pragma unroll
        for (int x = 0; x < 2; ++x) {
          if (!wait(&p_full[x][pb], pu & 1)) return false;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t bd = smem_desc(va + (4 * x + kk) * 2048, BOX, 1024, kLayoutSw128);
            mma_bf16_ts(tbase + COL_O + x * 128, tbase + COL_S + pb * 128 + x * 64 + kk * 8, bd, IDESC_O,
                        (first_of_unit && kk == 0) ? 0u : 1u);
          }
          tc_commit(&pv_done[x][pb]);
        }
        tc_commit(&v_empty[slot]);
        return true;
      };
      for (int u = blockIdx.x; u < units && ok && !abort_flag; u += gridDim.x, ++nunit) {
        int b, h, qt;
        unit_of(p, u, b, h, qt);
        qslot = nunit % QS;
        if (!wait(&q_full[qslot], (nunit / QS) & 1)) {
          ok = false;
          break;
        }
        const int t0 = tile;
        for (int kt = 0; kt <= qt && ok; ++kt, ++tile) {
          ok = scores(tile);
          if (ok && kt == qt) tc_commit(&q_empty[qslot]);  // the unit's last use of Q
          if (ok && kt > 0) ok = values(tile - 1, tile - 1 == t0);
        }
        if (ok) ok = values(tile - 1, tile - 1 == t0);
        if (ok) tc_commit(&o_ready);
      }
      if (!ok) abort_flag = 1;
    }
    __syncwarp();
  } else if (warp < 8) {
    // ------------------------------------------------------------------ softmax, half x of every tile's keys
    const int x = warp >> 2;
    const int row = tid & 127;  // query row within the tile = TMEM lane
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    const uint32_t col_o = tbase + lane_off + COL_O + x * 128;
    int tile = 0, nunit = 0;
    for (int u = blockIdx.x; u < units && !abort_flag; u += gridDim.x, ++nunit) {
      int b, h, qt;
      unit_of(p, u, b, h, qt);
      float m = -INFINITY, l = 0.f;
      for (int kt = 0; kt <= qt; ++kt, ++tile) {
        const int sb = tile & 1;
        if (!wait(&s_full[sb], (tile >> 1) & 1)) break;
        tc_fence_after();
        __syncwarp();
        const uint32_t scol = tbase + lane_off + COL_S + sb * 128 + x * 64;
        uint32_t raw[64];
        tmem_ld32_async(scol, raw);
        tmem_ld32_async(scol + 32, raw + 32);
        tmem_wait_ld();
        float v[64];
#pragma unroll
        for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(raw[i]);
        if (kt == qt) {  // the diagonal tile: keys past the query
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (x * 64 + i > row) v[i] = -INFINITY;
        }
        float part[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) part[j] = v[j];
#pragma unroll
        for (int i = 8; i < 64; ++i) part[i & 7] = fmaxf(part[i & 7], v[i]);
        const float tmax = fmaxf(fmaxf(fmaxf(part[0], part[1]), fmaxf(part[2], part[3])),
                                 fmaxf(fmaxf(part[4], part[5]), fmaxf(part[6], part[7]))) * p.qscale;
        // Raise the running max only when needed; then this half's O (built from earlier tiles) is rescaled. The
        // probabilities are formed first, so that the scores are dead while O is rescaled (register pressure).
        const float mnew = tmax > m + kRescale ? tmax : m;
        const bool rescale = mnew != m && kt > 0;
        const float mm = mnew == -INFINITY ? 0.f : mnew;  // a row with no key in this half yet: every p is 0
        uint32_t w[32];
        float ls[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) ls[j] = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float p0 = ex2(fmaf(v[2 * i], p.qscale, -mm));
          const float p1 = ex2(fmaf(v[2 * i + 1], p.qscale, -mm));
          ls[(2 * i) & 7] += p0;
          ls[(2 * i + 1) & 7] += p1;
          w[i] = pack_bf16x2(p0, p1);
        }
        if (__any_sync(0xffffffffu, rescale)) {
          if (!wait(&pv_done[x][(tile - 1) & 1], ((tile - 1) >> 1) & 1)) break;
          tc_fence_after();
          __syncwarp();
          const float sc = rescale ? ex2(m - mnew) : 1.f;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
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
        l += ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
        tmem_st32(scol, w);  // over this half's scores, which are in registers already
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[x][sb]);
      }
      if (abort_flag) break;
      // The unit's (max, sum) of this half for the epilogue, once the epilogue has read the previous unit's: a unit
      // of one or two tiles can be finished before that, and ml_full must not complete two phases ahead of its
      // waiter.
      if (nunit >= 1 && !wait(&ml_free, (nunit - 1) & 1)) break;
      ml_stash[x][row] = make_float2(m, l);
      mbar_arrive(&ml_full);
    }
  } else if (warp < 12) {
    // ------------------------------------------------------------------ epilogue (thread = query row)
    const int row = tid & 127;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    int nunit = 0;
    for (int u = blockIdx.x; u < units && !abort_flag; u += gridDim.x, ++nunit) {
      int b, h, qt;
      unit_of(p, u, b, h, qt);
      if (!wait(&o_ready, nunit & 1)) break;
      if (!wait(&ml_full, nunit & 1)) break;
      tc_fence_after();
      __syncwarp();
      const float2 e0 = ml_stash[0][row], e1 = ml_stash[1][row];
      mbar_arrive(&ml_free);
      const float mx = fmaxf(e0.x, e1.x);
      const float a0 = e0.y > 0.f ? ex2(e0.x - mx) : 0.f;
      const float a1 = e1.y > 0.f ? ex2(e1.x - mx) : 0.f;
      const float den = e0.y * a0 + e1.y * a1;
      const float inv = den > 0.f ? 1.f / den : 0.f;
      const float f0 = a0 * inv, f1 = a1 * inv;
      const int q = qt * BM + row;
      __nv_bfloat16* dst = p.out + (int64_t)b * p.out_sb + (int64_t)q * p.out_sw + (int64_t)h * p.out_sh;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        uint32_t r0[32], r1[32];
        tmem_ld32_async(tbase + lane_off + COL_O + c * 32, r0);
        tmem_ld32_async(tbase + lane_off + COL_O + 128 + c * 32, r1);
        tmem_wait_ld();
        if (q < p.width) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            uint32_t w4[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const int k = 8 * i + 2 * j;
              const float lo = fmaf(__uint_as_float(r0[k]), f0, __uint_as_float(r1[k]) * f1);
              const float hi = fmaf(__uint_as_float(r0[k + 1]), f0, __uint_as_float(r1[k + 1]) * f1);
              w4[j] = pack_bf16x2(lo, hi);
            }
            *reinterpret_cast<uint4*>(dst + c * 32 + i * 8) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&o_free);
    }
  }
  __syncthreads();
  if (abort_flag) {
    if (tid == 0) raise_status(p.status, kStatusTimeout);
    if (tid == W_MMA * 32) {
      tc_commit(&drain);  // every MMA the issuer thread issued has completed once this arrives
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
}

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
  p.group = prefill_group(a.batch * a.heads);
  p.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  p.out_sb = a.o_sb;
  p.out_sw = a.o_sw;
  p.out_sh = a.o_sh;
  p.status = a.status;
  const int units = a.batch * a.heads * p.qtiles;
  int grid = device_sm_count();
  if (grid > units) grid = units;
  if (grid <= 0) return cudaSuccess;
  return launch_dependent(prefill_kernel, dim3(grid), dim3(THREADS), (size_t)SMEM_BYTES, stream, qm, km, vm, p);
}

}  // namespace omni
