// Decode-time weight GEMMs on the 5th-generation tensor cores: y = epilogue(x . w^T), x [rows <= 64, k] (the step's
// tokens), w [n, k] (a layer's weights, read once per step: the work is HBM-bound weight streaming).
//
// Orientation: the weights take the MMA's M side (128-row tiles, A operand, K-major, 128-byte swizzle) and the
// tokens its N side (NT = rows rounded up to 16, B operand), so a 16 KB weight box feeds one tcgen05.mma of
// M=128 x N=NT x K=64; the fp32 accumulator tile [128 x NT] lives in TMEM (double-buffered). A stage holds KB
// consecutive 64-wide boxes of the same weight rows, so DRAM sees each row's KB * 128 bytes together.
//
// Schedule: persistent stream-K. The (weight tile, 64-wide K chunk) units, tile-major, are cut into one contiguous
// range per CTA (one CTA per SM), so every SM streams the same number of weight bytes whatever n. A tile whose
// chunks one CTA covers completely is finished by that CTA's epilogue. A tile cut between CTAs leaves an fp32 partial
// per contributor (slot 0: the CTA's first tile, slot 1: its last), summed in one fixed order whoever finishes the
// tile. A CTA's last range usually begins a tile whose other contributors worked on it first (at the start of their
// ranges): such a CTA watches the tile's arrival counter while its last MMAs run, sums the others' partials as soon
// as they are all in, and finishes the tile with its own accumulator as the last term -- so the end of a call
// carries no chain of global round trips. Otherwise the last contributor to arrive sums the slots. The finishing CTA
// sets the counter back to zero, so the counters are zero before and after every call and no second kernel is
// needed. Roles (192 threads): warp 0 TMA (weight boxes + token boxes per stage), warp 1 MMA issuer, warps 2-5
// epilogue (thread = weight row = TMEM lane).
//
// Cluster mode, for few long tiles (the 4096-wide projections: 32 tiles on 148 SMs, where stream-K would cut each
// tile between four or five CTAs that all finish at the end): a cluster of up to 4 CTAs per tile, each streaming a
// contiguous share of its chunks; after the role loops the partials are summed through distributed shared memory in
// rank order and each CTA writes out a share of the token rows.
//
// Launch: programmatic dependent. The first stages' weight boxes are requested before the dependency wait (the
// weights must not come from the kernel before), and the producer lets the next kernel launch once it has issued
// its last load.
//
// SwiGLU: the gate and inner rows of the same 64 outputs are two 64-row boxes of one 128-row tile (no weight copy),
// so the epilogue forms inner * silu(gate) within the tile.

#include <algorithm>
#include <cooperative_groups.h>
#include <cudaTypedefs.h>

#include "attention.cuh"
#include "common.cuh"
#include "tc.cuh"
#include "wgemm.cuh"

// Pipeline events of every CTA (entry, after the dependency wait, first load issued, first stage landed, last MMA
// issued, last accumulator handed over, epilogue done, exit), for a tracing harness that defines this hook before it
// includes this file; product builds compile it to nothing.
#ifndef OMNI_WG_EVENT
#define OMNI_WG_EVENT(args, ev) \
  do {                          \
  } while (0)
#endif

namespace omni {

namespace wg {

#ifndef OMNI_WGEMM_KB
#define OMNI_WGEMM_KB 4
#endif
constexpr int BM = 128;  // weight rows per tile
constexpr int BK = 64;   // K per box (one 128-byte swizzle row)
constexpr int KB = OMNI_WGEMM_KB;  // boxes per stage along K: each weight row gives KB * 128 contiguous bytes
constexpr int BKU = BK * KB;       // K per unit (chunk)
constexpr int W_BOX = BM * BK * 2;
constexpr int W_BYTES = KB * W_BOX;
// The first stages' weight boxes are requested before the dependency wait (the weights must not be written by the
// kernel launched just before on the same stream), and the next kernel may launch once every load is issued.
#ifndef OMNI_WGEMM_PREFETCH
#define OMNI_WGEMM_PREFETCH 1
#endif
#ifndef OMNI_WGEMM_EARLY_TRIGGER
#define OMNI_WGEMM_EARLY_TRIGGER 1
#endif
#ifndef OMNI_WGEMM_CLUSTER
#define OMNI_WGEMM_CLUSTER 1  // the per-tile cluster mode of launch_decode_gemm
#endif
#ifndef OMNI_WGEMM_STAGES
#define OMNI_WGEMM_STAGES (8 / OMNI_WGEMM_KB)
#endif
constexpr int STAGES = OMNI_WGEMM_STAGES;
constexpr int kMaxCluster = 4;  // CTAs per tile in cluster mode (the reduction is unrolled over this many ranks)
#ifndef OMNI_WGEMM_LATE_WATCH_NS
#define OMNI_WGEMM_LATE_WATCH_NS 3000
#endif
constexpr uint64_t kLateWatchNs = OMNI_WGEMM_LATE_WATCH_NS;  // the watch past the own accumulator (ns)
constexpr int THREADS = 192;

template <int NT>
struct Layout {
  static constexpr int X_BOX = NT * BK * 2;
  static constexpr int X_BYTES = KB * X_BOX;
  static constexpr int STAGE = W_BYTES + X_BYTES;  // a multiple of 1024 for NT in {16, 32, 48, 64}
  static constexpr int XCH_OFF = STAGES * STAGE;   // epilogue staging [NT][128] fp32
  static constexpr int BYTES = XCH_OFF + NT * BM * 4 + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * NT <= 32 ? 32 : (2 * NT <= 64 ? 64 : 128);
};

OMNI_DEV float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

OMNI_DEV int ld_relaxed_gpu(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// kGemmRope: a token's place, staged in shared memory once per CTA by the epilogue threads (thread m = token m):
// the offset of its cos/sin row (-1: position outside the table) and of its cache slot (-1: outside the cache).
struct TokenPlace {
  int64_t cs_off;
  int64_t cache_off;
};

OMNI_DEV void stage_tokens(const GemmArgs& a, int m, TokenPlace* place) {
  if (m >= a.rows) return;
  const RopeArgs& r = a.rope;
  const int64_t p = r.pos[m];
  const int64_t crow = r.slots ? r.slots[m] : m;
  const int64_t cp = r.cache_pos ? r.cache_pos[m] : p;
  const bool pos_ok = p >= 0 && p < r.cs_positions;
  const bool dst_ok = crow >= 0 && crow < r.cache_rows && cp >= 0 && cp < r.cache_len;
  if (!pos_ok || !dst_ok) raise_status(a.status, kStatusIndex);
  place[m].cs_off = pos_ok ? p * a.head_dim : -1;
  place[m].cache_off = dst_ok ? crow * r.s_kb + cp * r.s_ks : -1;
}

// Writes out token rows [m_lo, m_hi) of a finished tile held in `xch` ([NT][128] fp32: row m, column = the weight
// row of the tile) -- each thread 16-byte runs of 8 outputs of one token row, one vector store (and one vector
// residual load, all of a thread's loads issued before its first store, since y may be the residual) per 8 outputs.
// SwiGLU: columns 0..63 are the gate and 64..127 the inner products of outputs tile * 64 + c, each rounded to bf16
// before inner * silu(gate). The 128 threads call this together; it ends with the named barrier `bar`.
template <int NT, int MODE>
OMNI_DEV void finish_rows(const GemmArgs& a, int tile, int row, const float* xch, int m_lo, int m_hi, int bar) {
  constexpr int WIDTH = MODE == kGemmSwiglu ? 64 : BM;  // outputs of one tile
  constexpr int RUNS = WIDTH / 8;                       // 16-byte runs per token row
  constexpr int MAXK = (NT * RUNS + 127) / 128;         // runs per thread
  const int64_t col0 = (int64_t)tile * WIDTH;
  const int cols = (int)min((int64_t)WIDTH, (int64_t)a.n - col0);
  const bool vec_y = (a.ld_y & 7) == 0 && (reinterpret_cast<uintptr_t>(a.y) & 15) == 0;
  const bool vec_r =
      MODE != kGemmResidual || ((a.ld_res & 7) == 0 && (reinterpret_cast<uintptr_t>(a.residual) & 15) == 0);
  const int runs = (m_hi - m_lo) * RUNS;
#pragma unroll 1  // compact: see the epilogue's finish below
  for (int k = 0; k < MAXK; ++k) {
    const int c = row + 128 * k, m = m_lo + c / RUNS, j0 = (c % RUNS) * 8;
    if (c >= runs) break;
    uint4 res = make_uint4(0u, 0u, 0u, 0u);
    if (MODE == kGemmResidual) {
      const __nv_bfloat16* rsrc = a.residual + (int64_t)m * a.ld_res + col0 + j0;
      if (vec_r && j0 + 8 <= cols) {
        res = *reinterpret_cast<const uint4*>(rsrc);
      } else {
        __nv_bfloat16* r8 = reinterpret_cast<__nv_bfloat16*>(&res);
        for (int q = 0; q < 8; ++q)
          if (j0 + q < cols) r8[q] = rsrc[q];
      }
    }
    const float4* src = reinterpret_cast<const float4*>(xch + m * BM + j0);
    float v[8];
    if (MODE == kGemmSwiglu) {
      const float4 g0 = src[0], g1 = src[1], u0 = src[16], u1 = src[17];  // inner products: 64 columns on
      const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
      const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float gq = bf16r(g[q]);
        // silu(g) = g / (1 + e^-g); the fast divide's few-ulp error is far below the bf16 rounding that follows
        const float sq = bf16r(__fdividef(gq, 1.f + __expf(-gq)));
        v[q] = bf16r(u[q]) * sq;
      }
    } else {
      const float4 v0 = src[0], v1 = src[1];
      v[0] = v0.x, v[1] = v0.y, v[2] = v0.z, v[3] = v0.w, v[4] = v1.x, v[5] = v1.y, v[6] = v1.z, v[7] = v1.w;
      if (MODE == kGemmResidual) {
        const __nv_bfloat16* r8 = reinterpret_cast<const __nv_bfloat16*>(&res);
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] += __bfloat162float(r8[q]);
      }
    }
    uint4 out;
    __nv_bfloat16* o8 = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
    for (int q = 0; q < 8; ++q) o8[q] = __float2bfloat16_rn(v[q]);
    __nv_bfloat16* dst = a.y + (int64_t)m * a.ld_y + col0 + j0;
    if (vec_y && j0 + 8 <= cols) {
      *reinterpret_cast<uint4*>(dst) = out;
    } else {
      for (int q = 0; q < 8; ++q)
        if (j0 + q < cols) dst[q] = o8[q];
    }
  }
  named_sync(bar, 128);  // xch free again
}

// The epilogue of one finished weight tile: thread `row` (0..127) holds acc[m] of token m for weight row
// tile * 128 + row (SwiGLU: rows 0..63 gate, 64..127 inner of outputs tile * 64 + row % 64). `xch` is shared memory
// of the 128 participating threads, which all call this together (named barrier `bar`).
template <int NT, int MODE>
OMNI_DEV void finish_tile(const GemmArgs& a, int tile, int row, const float (&acc)[NT], float* xch, int bar) {
  if constexpr (MODE == kGemmRope) {
    // The tile's 128 features are dims d0..d0+127 of one head h of section q / k / v (128 divides the head_dim);
    // thread `row` holds dim d0 + row, so a rotation pair (2j, 2j + 1) is two neighbouring lanes (one shuffle).
    // Each product is rounded to bf16 first, as the GEMM's output would be, then rotated in fp32 with the
    // non-contracting products of rope_kv.cu (omniasr_trt/modeling.py:301-306); cos/sin pairs are fetched for a
    // batch of tokens at a time ahead of their use. The rotated tile is staged as bf16 [NT][128] in shared memory after
    // the tokens' places (staged once per CTA by stage_tokens), then written as 16-byte runs of one token's dims:
    // q always (zero for a position outside the table), k only with a rotation and a cache slot, v with a slot.
    const RopeArgs& r = a.rope;
    const TokenPlace* place = reinterpret_cast<const TokenPlace*>(xch);
    __nv_bfloat16* stage =
        reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<char*>(xch) + kGemmMaxRows * sizeof(TokenPlace));
    const int per = r.heads * a.head_dim;
    const int f0 = tile * BM, part = f0 / per, h = (f0 - part * per) / a.head_dim;
    const int d0 = f0 - part * per - h * a.head_dim;
    const bool odd = row & 1;
    const float* cs_base = r.cs + ((d0 + row) & ~1);
    constexpr int HALF = NT == 64 ? 16 : NT / 2;  // tokens per batch of cos/sin loads (64: a quarter, for registers)
#pragma unroll
    for (int m0 = 0; m0 < NT; m0 += HALF) {
      float2 cs[HALF];
      bool rot[HALF];
#pragma unroll
      for (int j = 0; j < HALF; ++j) {
        const int m = m0 + j;
        const int64_t so = m < a.rows && part < 2 ? place[m].cs_off : -1;
        rot[j] = so >= 0;
        cs[j] = rot[j] ? __ldg(reinterpret_cast<const float2*>(cs_base + so)) : make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int j = 0; j < HALF; ++j) {
        const int m = m0 + j;
        const float x = bf16r(acc[m]);
        const float other = __shfl_xor_sync(0xffffffffu, x, 1);
        const float re = odd ? other : x, im = odd ? x : other;
        const float y = part == 2 ? x
                        : !rot[j] ? 0.f
                        : odd     ? __fadd_rn(__fmul_rn(re, cs[j].y), __fmul_rn(im, cs[j].x))
                                  : __fsub_rn(__fmul_rn(re, cs[j].x), __fmul_rn(im, cs[j].y));
        stage[m * BM + row] = __float2bfloat16_rn(y);
      }
    }
    named_sync(bar, 128);
    __nv_bfloat16* q_out = reinterpret_cast<__nv_bfloat16*>(r.q_out);
    __nv_bfloat16* cache = reinterpret_cast<__nv_bfloat16*>(part == 1 ? r.k_cache : r.v_cache);
    const bool vec = part == 0 ? (reinterpret_cast<uintptr_t>(q_out) & 15) == 0
                               : (reinterpret_cast<uintptr_t>(cache) & 15) == 0 &&
                                     ((r.s_kb | r.s_kh | r.s_ks) & 7) == 0;
    constexpr int RUNS = BM / 8;
    constexpr int MAXK = (NT * RUNS + 127) / 128;
#pragma unroll 1
    for (int k = 0; k < MAXK; ++k) {
      const int c = row + 128 * k, m = c / RUNS, j0 = (c % RUNS) * 8;
      if (c >= a.rows * RUNS) break;
      __nv_bfloat16* dst;
      if (part == 0) {
        dst = q_out + (int64_t)m * per + (int64_t)h * a.head_dim + d0 + j0;
      } else {
        const int64_t co = place[m].cache_off;
        if (co < 0 || (part == 1 && place[m].cs_off < 0)) continue;
        dst = cache + co + (int64_t)h * r.s_kh + d0 + j0;
      }
      const uint4 v = *reinterpret_cast<const uint4*>(stage + m * BM + j0);
      if (vec) {
        *reinterpret_cast<uint4*>(dst) = v;
      } else {
        const __nv_bfloat16* v8 = reinterpret_cast<const __nv_bfloat16*>(&v);
#pragma unroll
        for (int q = 0; q < 8; ++q) dst[q] = v8[q];
      }
    }
    named_sync(bar, 128);  // the stage is free again
  } else {
    // Store / residual / SwiGLU: the tile goes through shared memory (`xch`, [NT][128] fp32, thread `row` writes
    // column `row`), then finish_rows writes it out.
#pragma unroll
    for (int m = 0; m < NT; ++m) xch[m * BM + row] = acc[m];
    named_sync(bar, 128);
    finish_rows<NT, MODE>(a, tile, row, xch, 0, a.rows, bar);
  }
}

template <int NT, int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    wgemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap, const GemmArgs a) {
  using L = Layout<NT>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], acc_full[2], acc_free[2], drain;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int abort_flag;
  __shared__ volatile int issued;
  __shared__ int last_flag_s;
  int* last_flag = &last_flag_s;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) OMNI_WG_EVENT(a, 0);
  const int64_t total = (int64_t)a.tiles * a.chunks;
  // Stream-K: one contiguous range of `per` units per CTA. Cluster mode (a.cluster = S > 1): cluster i (CTAs
  // S * i .. S * i + S - 1, rank = blockIdx.x % S) owns tile i, each CTA a contiguous 1/S of its chunks; the host
  // chooses it only when every CTA gets at least one chunk, so no CTA of a cluster leaves early.
  const int S = a.cluster;
  const int64_t u0 = S > 1 ? (int64_t)(blockIdx.x / S) * a.chunks + (blockIdx.x % S) * a.chunks / S
                           : (int64_t)blockIdx.x * a.per;
  const int64_t u1 = S > 1 ? (int64_t)(blockIdx.x / S) * a.chunks + (blockIdx.x % S + 1) * a.chunks / S
                           : min(total, u0 + a.per);
  if (u0 >= u1) return;  // uniform over the CTA (never in cluster mode)

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_free[b], 128);
    }
    mbar_init(&drain, 1);
    mbar_fence_init();
    abort_flag = 0;
    issued = 0;
  }
  if (warp == 0) tmem_alloc(&tmem_base, L::TMEM_COLS);
  if (warp == 1 && lane == 0) {
    prefetch_tmap(&wmap);
    prefetch_tmap(&xmap);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();

  // The weight boxes of stage i (unit u) and its token boxes; stage i's `full` barrier expects both.
  auto load_w = [&](int i, int64_t u) {
    const int t = (int)(u / a.chunks), c = (int)(u % a.chunks);
    unsigned char* st = smem + (i % STAGES) * L::STAGE;
    uint64_t* bar = &full[i % STAGES];
    mbar_arrive_expect_tx(bar, L::STAGE);
#pragma unroll
    for (int j = 0; j < KB; ++j) {  // the weight boxes back to back: each row's KB * 128 bytes together
      const int kx = c * BKU + j * BK;
      if (MODE == kGemmSwiglu) {
        tma_load_2d(st + j * W_BOX, &wmap, kx, t * 64, bar);                   // gate rows
        tma_load_2d(st + j * W_BOX + W_BOX / 2, &wmap, kx, a.n + t * 64, bar);  // inner rows
      } else {
        tma_load_2d(st + j * W_BOX, &wmap, kx, t * BM, bar);
      }
    }
  };
  auto load_x = [&](int i, int64_t u) {
    const int c = (int)(u % a.chunks);
    unsigned char* st = smem + (i % STAGES) * L::STAGE;
#pragma unroll
    for (int j = 0; j < KB; ++j)
      tma_load_2d(st + W_BYTES + j * L::X_BOX, &xmap, c * BKU + j * BK, 0, &full[i % STAGES]);
  };
  // The weights do not depend on the kernel before: the first stages' weight boxes are requested before the
  // dependency wait, so their latency overlaps that kernel's tail.
  int pre = 0;
#if OMNI_WGEMM_PREFETCH
  if (warp == 0 && lane == 0) {
    for (; pre < STAGES && u0 + pre < u1; ++pre) load_w(pre, u0 + pre);
    OMNI_WG_EVENT(a, 2);
  }
#endif
  grid_dependency_wait();  // the tokens come from the kernel before (launched as a programmatic dependent)
  if (tid == 0) OMNI_WG_EVENT(a, 1);
  const uint32_t tbase = tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int i = 0;
      for (; i < pre; ++i) load_x(i, u0 + i);  // the token boxes of the prefetched stages, whatever happens next
      issued = pre;
      for (int64_t u = u0 + pre; u < u1 && !abort_flag; ++u, ++i) {
        const int s = i % STAGES, use = i / STAGES;
        if (use >= 1 && !mbar_wait(&empty[s], (use - 1) & 1)) {
          abort_flag = 1;
          break;
        }
        load_w(i, u);
        load_x(i, u);
        if (i == 0) OMNI_WG_EVENT(a, 2);
        issued = i + 1;
      }
#if OMNI_WGEMM_EARLY_TRIGGER
      grid_launch_dependents();  // every load issued: the next kernel's blocks may take free SMs and prefetch
#endif
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t IDESC = idesc_bf16(BM, NT, 0, 0);
      int i = 0, seg = 0;
      bool ok = true;
      for (int64_t u = u0; u < u1 && ok && !abort_flag; ++u, ++i) {
        const int c = (int)(u % a.chunks);
        const bool seg_first = u == u0 || c == 0;
        const bool seg_last = u == u1 - 1 || c == a.chunks - 1;
        const int buf = seg & 1;
        if (seg_first && seg >= 2 && !mbar_wait(&acc_free[buf], ((seg >> 1) - 1) & 1)) {
          ok = false;
          break;
        }
        const int s = i % STAGES;
        if (!mbar_wait(&full[s], (i / STAGES) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (i == 0) OMNI_WG_EVENT(a, 3);
        const uint32_t wa = smem_addr(smem + s * L::STAGE), xa = wa + W_BYTES;
#pragma unroll
        for (int kk = 0; kk < BKU / 16; ++kk) {
          const uint64_t ad = smem_desc(wa + (kk >> 2) * W_BOX + (kk & 3) * 32, 16, 1024, kLayoutSw128);
          const uint64_t bd = smem_desc(xa + (kk >> 2) * L::X_BOX + (kk & 3) * 32, 16, 1024, kLayoutSw128);
          mma_bf16_ss(tbase + buf * NT, ad, bd, IDESC, (seg_first && kk == 0) ? 0u : 1u);
        }
        tc_commit(&empty[s]);
        if (seg_last) {
          tc_commit(&acc_full[buf]);
          ++seg;
        }
      }
      if (!ok) abort_flag = 1;
      OMNI_WG_EVENT(a, 4);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue (thread = weight row)
    const int row = 32 * (warp & 3) + lane;
    const uint32_t lane_off = (uint32_t)(32 * (warp & 3)) << 16;
    float* xch = reinterpret_cast<float*>(smem + L::XCH_OFF);
    if (MODE == kGemmRope) {  // the tokens' places, once per CTA (the exchange area is free in this mode)
      if (row < kGemmMaxRows) stage_tokens(a, row, reinterpret_cast<TokenPlace*>(xch));
      named_sync(3, 128);
    }
    int seg = 0;
    for (int64_t u = u0; u < u1; ++seg) {
      const int t = (int)(u / a.chunks), c0 = (int)(u % a.chunks);
      const int64_t seg_end = min(u1, (int64_t)(t + 1) * a.chunks);  // exclusive
      const bool whole = c0 == 0 && seg_end == (int64_t)(t + 1) * a.chunks;
      const int buf = seg & 1;
      if (S > 1) {
        // Cluster mode: the CTA's one range; its partial goes to the (now idle) stage area, [NT][128] fp32, for the
        // cluster's reduction after the role loops.
        if (!mbar_wait(&acc_full[buf], (seg >> 1) & 1)) abort_flag = 1;
        tc_fence_after();
        __syncwarp();
        float acc[NT];
#pragma unroll
        for (int c = 0; c < NT; c += 16) tmem_ld16(tbase + lane_off + buf * NT + c, acc + c);
        tc_fence_before();
        mbar_arrive(&acc_free[buf]);
        float* part = reinterpret_cast<float*>(smem);
#pragma unroll
        for (int m = 0; m < NT; ++m) part[m * BM + row] = acc[m];
        u = seg_end;
        continue;
      }
      // A split tile's contributors are CTAs b0..b1; each leaves its fp32 partial in its own slot and the tile is
      // summed in one fixed order, p[b1] + p[b1 - 1] + ... + p[b0], whoever finishes it, so results do not depend
      // on timing. The contributor that begins the tile (b0: the last range of its CTA, while the others met the
      // tile at the start of theirs) watches the tile's counter while its accumulator is still being computed; once
      // every other contributor has arrived it sums their partials ahead of its own and finishes the tile with its
      // accumulator as the last term, without publishing it -- so the end of a call carries no chain of global
      // round trips. Otherwise the last contributor to arrive sums the slots.
      const int64_t tc0 = (int64_t)t * a.chunks;
      const int me = blockIdx.x;
      const int b0 = (int)(tc0 / a.per), b1 = (int)((tc0 + a.chunks - 1) / a.per);
      auto slot_of = [&](int b) -> const float4* {
        const int sl = t == (int)(((int64_t)b * a.per) / a.chunks) ? 0 : 1;
        return reinterpret_cast<const float4*>(a.part) + ((int64_t)(b * 2 + sl) * (NT / 4)) * BM + row;
      };
      float others[NT];
      bool early = false;
      if (!whole && me == b0) {
        // The watch goes on for a short while after the own accumulator is ready: a contributor that covers the
        // middle of the tile finishes at about the same time, and one more wait for its arrival is shorter than
        // the chain of the arrive-and-sum path.
        const uint64_t t0 = global_ns();
        uint64_t t_acc = 0;
        int f = 0;
        do {
          if (row == 0) {
            // a relaxed poll; the fence below orders the partial loads after the arrivals it saw
            int v = ld_relaxed_gpu(&a.counters[t]) == b1 - b0 ? 1 : 0;
            if (!v && (t_acc != 0 || mbar_test_wait(&acc_full[buf], (seg >> 1) & 1))) {
              const uint64_t now = global_ns();
              if (t_acc == 0) t_acc = now;
              if (now - t_acc > kLateWatchNs) v = 2;
            }
            if (!v && global_ns() - t0 > kWaitLimitNs) v = 3;
            *last_flag = v;
          }
          named_sync(2, 128);
          f = *last_flag;
          named_sync(2, 128);
          if (f == 0 && row == 0) __nanosleep(200);
        } while (f == 0);
        OMNI_WG_EVENT(a, 8 + f);
        if (f == 3) abort_flag = 1;
        early = f == 1;
        if (early) {
          __threadfence();
          for (int b = b1; b > b0; --b) {
            const float4* src = slot_of(b);
#pragma unroll
            for (int m = 0; m < NT; m += 4) {
              const float4 v = __ldcg(src + (m / 4) * BM);  // other CTAs' stores: from L2
              if (b == b1) {
                others[m] = v.x, others[m + 1] = v.y, others[m + 2] = v.z, others[m + 3] = v.w;
              } else {
                others[m] += v.x, others[m + 1] += v.y, others[m + 2] += v.z, others[m + 3] += v.w;
              }
            }
          }
        }
      }
      if (!mbar_wait(&acc_full[buf], (seg >> 1) & 1)) abort_flag = 1;
      if (tid == 64 && seg_end == u1) OMNI_WG_EVENT(a, 5);
      tc_fence_after();
      __syncwarp();
      float acc[NT];
#pragma unroll
      for (int c = 0; c < NT; c += 16) tmem_ld16(tbase + lane_off + buf * NT + c, acc + c);
      tc_fence_before();
      mbar_arrive(&acc_free[buf]);
      // Whole tiles, early finishes and last arrivals all end in the one finish_tile below: the kernel's code stays
      // small, and code size matters here (the epilogue runs once or twice per call, and a larger body slowed the
      // weight stream of the other warps as well).
      bool finish = whole;
      if (!whole && early) {
#pragma unroll
        for (int m = 0; m < NT; ++m) acc[m] = others[m] + acc[m];
        finish = true;
      } else if (!whole) {
        float4* dst = const_cast<float4*>(slot_of(me));
#pragma unroll
        for (int m = 0; m < NT; m += 4) dst[(m / 4) * BM] = make_float4(acc[m], acc[m + 1], acc[m + 2], acc[m + 3]);
        __threadfence();
        named_sync(2, 128);
        if (row == 0) *last_flag = atomicAdd(&a.counters[t], 1) == b1 - b0;
        named_sync(2, 128);
        if (tid == 64) OMNI_WG_EVENT(a, 14);
        finish = *last_flag;
        if (finish) {
          __threadfence();
          // Two slots per round trip, summed in the fixed order.
          for (int b = b1; b >= b0; b -= 2) {
            const float4* s0 = slot_of(b);
            const float4* s1 = slot_of(b > b0 ? b - 1 : b);
            float4 v0[NT / 4], v1[NT / 4];
#pragma unroll
            for (int m = 0; m < NT / 4; ++m) {
              v0[m] = __ldcg(s0 + m * BM);
              v1[m] = __ldcg(s1 + m * BM);
            }
#pragma unroll
            for (int m = 0; m < NT / 4; ++m) {
              if (b == b1) {
                acc[4 * m] = v0[m].x, acc[4 * m + 1] = v0[m].y, acc[4 * m + 2] = v0[m].z, acc[4 * m + 3] = v0[m].w;
              } else {
                acc[4 * m] += v0[m].x, acc[4 * m + 1] += v0[m].y, acc[4 * m + 2] += v0[m].z, acc[4 * m + 3] += v0[m].w;
              }
              if (b > b0) {
                acc[4 * m] += v1[m].x, acc[4 * m + 1] += v1[m].y, acc[4 * m + 2] += v1[m].z, acc[4 * m + 3] += v1[m].w;
              }
            }
          }
        }
      }
      if (finish) {
        if (tid == 64) OMNI_WG_EVENT(a, 12);
        finish_tile<NT, MODE>(a, t, row, acc, xch, 1);
        if (tid == 64) OMNI_WG_EVENT(a, 13);
        if (!whole && row == 0) a.counters[t] = 0;  // zero again for the next call
      }
      u = seg_end;
      if (abort_flag) break;
    }
    if (tid == 64) OMNI_WG_EVENT(a, 6);
  }
  __syncthreads();
  if (abort_flag) {
    if (tid == 0) raise_status(a.status, kStatusTimeout);
    if (tid == 32) {
      tc_commit(&drain);
      mbar_wait(&drain, 0);
    }
  }
  __syncthreads();
  if (abort_flag && tid == 0) {
    // Let the latest load of every stage land before the shared memory goes away.
    for (int i = issued > STAGES ? issued - STAGES : 0; i < issued; ++i) mbar_wait(&full[i % STAGES], (i / STAGES) & 1);
  }
  if (S > 1) {
    // Cluster mode: the S partials of the tile are summed through distributed shared memory, rank S - 1 first
    // (a fixed order), each CTA for its share of the token rows, which it then writes out.
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    if (tid == 64) OMNI_WG_EVENT(a, 11);
    cluster.sync();  // every partial of the cluster in place
    if (tid == 64) OMNI_WG_EVENT(a, 12);
    if (warp >= 2) {
      const int row = 32 * (warp & 3) + lane;
      const int q = (int)cluster.block_rank();
      const int m_lo = q * a.rows / S, m_hi = (q + 1) * a.rows / S;
      float* xch = reinterpret_cast<float*>(smem + L::XCH_OFF);
      // Thread = (one of 4 token rows, 4 consecutive weight rows); two token rows per pass, every rank's float4 of
      // both requested before any is summed, so a pass costs one distributed-shared-memory round trip.
      constexpr int MAXS = kMaxCluster;
      const int g = row & 31, mo = row >> 5;
      const float4* src[MAXS];
#pragma unroll
      for (int j = 0; j < MAXS; ++j)
        src[j] = reinterpret_cast<const float4*>(cluster.map_shared_rank(reinterpret_cast<float*>(smem), j < S ? j : 0));
      for (int m0 = m_lo + mo; m0 < m_hi; m0 += 8) {
        const int m1 = m0 + 4;
        const bool two = m1 < m_hi;
        float4 v0[MAXS], v1[MAXS];
#pragma unroll
        for (int j = 0; j < MAXS; ++j) {
          if (j < S) {
            v0[j] = src[j][m0 * (BM / 4) + g];
            if (two) v1[j] = src[j][m1 * (BM / 4) + g];
          }
        }
        float4 s0 = make_float4(0.f, 0.f, 0.f, 0.f), s1 = s0;
        bool first = true;
#pragma unroll
        for (int j = MAXS - 1; j >= 0; --j) {  // rank S - 1 first: a fixed order
          if (j < S) {
            if (first) {
              s0 = v0[j], s1 = v1[j];
            } else {
              s0.x += v0[j].x, s0.y += v0[j].y, s0.z += v0[j].z, s0.w += v0[j].w;
              s1.x += v1[j].x, s1.y += v1[j].y, s1.z += v1[j].z, s1.w += v1[j].w;
            }
            first = false;
          }
        }
        reinterpret_cast<float4*>(xch)[m0 * (BM / 4) + g] = s0;
        if (two) reinterpret_cast<float4*>(xch)[m1 * (BM / 4) + g] = s1;
      }
      named_sync(1, 128);
      if (tid == 64) OMNI_WG_EVENT(a, 13);
      finish_rows<NT, MODE>(a, (int)(u0 / a.chunks), row, xch, m_lo, m_hi, 1);
      if (tid == 64) OMNI_WG_EVENT(a, 14);
    }
    cluster.sync();  // no CTA leaves while the others read its partial
    if (tid == 64) OMNI_WG_EVENT(a, 15);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, L::TMEM_COLS);
  }
  if (tid == 0) OMNI_WG_EVENT(a, 7);
  grid_launch_dependents();
}

bool make_map_2d(CUtensorMap* map, const void* base, int64_t cols, int64_t rows, int64_t ld, int box_cols,
                 int box_rows) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NT, int MODE>
cudaError_t launch_t(const CUtensorMap& wm, const CUtensorMap& xm, const GemmArgs& a, cudaStream_t stream) {
  using L = Layout<NT>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(wgemm_kernel<NT, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  if (a.cluster <= 1)
    return launch_dependent(wgemm_kernel<NT, MODE>, dim3((unsigned)a.grid), dim3(THREADS), (size_t)L::BYTES, stream,
                            wm, xm, a);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)a.grid);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = (size_t)L::BYTES;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = (unsigned)a.cluster;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, wgemm_kernel<NT, MODE>, wm, xm, a);
}

template <int NT>
cudaError_t launch_mode(const CUtensorMap& wm, const CUtensorMap& xm, const GemmArgs& a, cudaStream_t stream) {
  switch (a.mode) {
    case kGemmStore:
      return launch_t<NT, kGemmStore>(wm, xm, a, stream);
    case kGemmResidual:
      return launch_t<NT, kGemmResidual>(wm, xm, a, stream);
    case kGemmSwiglu:
      return launch_t<NT, kGemmSwiglu>(wm, xm, a, stream);
    case kGemmRope:
      return launch_t<NT, kGemmRope>(wm, xm, a, stream);
    default:
      return cudaErrorInvalidValue;
  }
}

}  // namespace wg

int gemm_token_tile(int rows) { return rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 48 ? 48 : 64; }

int gemm_tiles(int n, int mode) { return mode == kGemmSwiglu ? (n + 63) / 64 : (n + wg::BM - 1) / wg::BM; }

// A fixed size, so that calls of different shapes sharing a workspace agree on where the counters end.
size_t gemm_counter_bytes(int n, int mode) {
  (void)n;
  (void)mode;
  return (size_t)kGemmMaxTiles * sizeof(int);
}

size_t gemm_workspace_bytes(int rows, int n, int k, int mode) {
  (void)k;
  return gemm_counter_bytes(n, mode) + (size_t)device_sm_count() * 2 * wg::BM * gemm_token_tile(rows) * sizeof(float);
}

cudaError_t launch_decode_gemm(const void* x, int64_t ldx, const void* w, int64_t ldw, GemmArgs a, void* workspace,
                               size_t workspace_bytes, cudaStream_t stream) {
  using namespace wg;
  const int nt = gemm_token_tile(a.rows);
  const int wrows = a.mode == kGemmSwiglu ? 2 * a.n : a.n;
  CUtensorMap wm, xm;
  if (!make_map_2d(&wm, w, a.k, wrows, ldw, BK, a.mode == kGemmSwiglu ? 64 : BM) ||
      !make_map_2d(&xm, x, a.k, a.rows, ldx, BK, nt))
    return cudaErrorInvalidValue;
  a.tiles = gemm_tiles(a.n, a.mode);
  a.chunks = (a.k + BKU - 1) / BKU;
  const int64_t total = (int64_t)a.tiles * a.chunks;
  const int sms = device_sm_count();
  int grid = sms;
  if (grid > total) grid = (int)total;
  a.per = (total + grid - 1) / grid;
  a.grid = (int)((total + a.per - 1) / a.per);
  // Few, long tiles (the 4096-wide projections: 32 tiles on 148 SMs): stream-K would cut each tile between four or
  // five CTAs that all finish at the end of the call, leaving a chain of global round trips to whichever is last.
  // Instead a cluster of S CTAs takes each tile and reduces it through distributed shared memory -- when that still
  // keeps three quarters of the SMs streaming.
  a.cluster = 1;
  if (OMNI_WGEMM_CLUSTER && a.mode != kGemmRope) {
    int S = std::min(kMaxCluster, sms / a.tiles);
    while (S > 1 && a.chunks < S) --S;
    if (S > 1 && 4 * a.tiles * S >= 3 * sms) {
      a.cluster = S;
      a.grid = a.tiles * S;
    }
  }
  const size_t cbytes = gemm_counter_bytes(a.n, a.mode);
  if (workspace_bytes < cbytes + (size_t)a.grid * 2 * BM * nt * sizeof(float)) return cudaErrorInvalidValue;
  a.counters = static_cast<int*>(workspace);
  a.part = reinterpret_cast<float*>(static_cast<char*>(workspace) + cbytes);
  switch (nt) {
    case 16:
      return launch_mode<16>(wm, xm, a, stream);
    case 32:
      return launch_mode<32>(wm, xm, a, stream);
    case 48:
      return launch_mode<48>(wm, xm, a, stream);
    default:
      return launch_mode<64>(wm, xm, a, stream);
  }
}

}  // namespace omni
