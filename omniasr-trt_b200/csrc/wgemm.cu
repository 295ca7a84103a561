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
// chunks one CTA covers completely is finished by that CTA's epilogue; a tile cut between CTAs leaves an fp32
// partial per CTA (slot 0: the CTA's first tile, slot 1: its last), and the last of those CTAs to finish (a per-tile
// arrival counter in the workspace) sums them and runs the same epilogue, then sets the counter back to zero -- so
// the counters are zero before and after every call, and no second kernel is needed. Roles (192 threads): warp 0 TMA (weight box + token box per stage, 8-stage ring), warp 1 MMA
// issuer, warps 2-5 epilogue (thread = weight row = TMEM lane).
//
// SwiGLU: the gate and inner rows of the same 64 outputs are two 64-row boxes of one 128-row tile (no weight copy),
// so the epilogue forms inner * silu(gate) within the tile.

#include <cudaTypedefs.h>

#include "attention.cuh"
#include "common.cuh"
#include "tc.cuh"
#include "wgemm.cuh"

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
#ifndef OMNI_WGEMM_STAGES
#define OMNI_WGEMM_STAGES (8 / OMNI_WGEMM_KB)
#endif
constexpr int STAGES = OMNI_WGEMM_STAGES;
constexpr int THREADS = 192;

template <int NT>
struct Layout {
  static constexpr int X_BOX = NT * BK * 2;
  static constexpr int X_BYTES = KB * X_BOX;
  static constexpr int STAGE = W_BYTES + X_BYTES;  // a multiple of 1024 for NT in {16, 32, 48, 64}
  static constexpr int XCH_OFF = STAGES * STAGE;   // SwiGLU exchange [64][NT] fp32
  static constexpr int BYTES = XCH_OFF + 64 * NT * 4 + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * NT <= 32 ? 32 : (2 * NT <= 64 ? 64 : 128);
};

OMNI_DEV float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

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

// The epilogue of one finished weight tile: thread `row` (0..127) holds acc[m] of token m for weight row
// tile * 128 + row (SwiGLU: rows 0..63 gate, 64..127 inner of outputs tile * 64 + row % 64). `xch` is shared memory
// of the 128 participating threads, which all call this together (named barrier `bar`).
template <int NT, int MODE>
OMNI_DEV void finish_tile(const GemmArgs& a, int tile, int row, const float (&acc)[NT], float* xch, int bar) {
  if (MODE == kGemmSwiglu) {
    if (row >= 64) {
#pragma unroll
      for (int m = 0; m < NT; ++m) xch[(row - 64) * NT + m] = acc[m];
    }
    named_sync(bar, 128);
    if (row < 64) {
      const int f = tile * 64 + row;
      if (f < a.n) {
#pragma unroll
        for (int m = 0; m < NT; ++m) {
          if (m < a.rows) {
            const float g = bf16r(acc[m]);
            const float u = bf16r(xch[row * NT + m]);
            const float s = bf16r(g / (1.f + __expf(-g)));
            a.y[(int64_t)m * a.ld_y + f] = __float2bfloat16_rn(u * s);
          }
        }
      }
    }
    named_sync(bar, 128);  // xch free again
    return;
  }
  if (MODE == kGemmRope) {
    // Feature f = tile * 128 + row is head dim d of head h of section q / k / v (128 divides the head_dim, so a
    // rotation pair (2j, 2j + 1) never straddles two tiles: its partner is the neighbouring lane). Each product is
    // rounded to bf16 first, as the GEMM's output would be, then rotated in fp32 with the non-contracting products
    // of rope_kv.cu (omniasr_trt/modeling.py:301-306). The tokens' places come from shared memory (`xch`, staged by
    // stage_tokens); their cos/sin pairs are fetched eight tokens at a time ahead of the stores.
    const RopeArgs& r = a.rope;
    const TokenPlace* place = reinterpret_cast<const TokenPlace*>(xch);
    const int f = tile * BM + row;
    const int per = r.heads * a.head_dim;
    const int part = f / per, h = (f - part * per) / a.head_dim, d = f - part * per - h * a.head_dim;
    const bool odd = d & 1;
    const float* cs_base = r.cs + (d & ~1);
    __nv_bfloat16* q_out = reinterpret_cast<__nv_bfloat16*>(r.q_out) + (int64_t)h * a.head_dim + d;
    const int64_t head_off = (int64_t)h * r.s_kh + d;
#pragma unroll
    for (int m0 = 0; m0 < NT; m0 += 8) {
      float2 cs[8];
      int64_t coff[8];
      bool rot[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int m = m0 + j;
        const int64_t so = m < a.rows && part < 2 ? place[m].cs_off : -1;
        coff[j] = m < a.rows ? place[m].cache_off : -1;
        rot[j] = so >= 0;
        cs[j] = rot[j] ? __ldg(reinterpret_cast<const float2*>(cs_base + so)) : make_float2(0.f, 0.f);
        if (so < 0) coff[j] = part < 2 ? -1 : coff[j];  // no k without a rotation (v needs none)
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int m = m0 + j;
        const float x = bf16r(acc[m]);
        const float other = __shfl_xor_sync(0xffffffffu, x, 1);
        if (m >= a.rows || f >= a.n) continue;
        if (part == 2) {
          if (coff[j] >= 0) reinterpret_cast<__nv_bfloat16*>(r.v_cache)[coff[j] + head_off] = __float2bfloat16_rn(x);
          continue;
        }
        const float re = odd ? other : x, im = odd ? x : other;
        const float y = !rot[j] ? 0.f
                        : odd   ? __fadd_rn(__fmul_rn(re, cs[j].y), __fmul_rn(im, cs[j].x))
                                : __fsub_rn(__fmul_rn(re, cs[j].x), __fmul_rn(im, cs[j].y));
        if (part == 0) {
          q_out[(int64_t)m * r.heads * a.head_dim] = __float2bfloat16_rn(y);  // zero for a position outside the table
        } else if (coff[j] >= 0) {
          reinterpret_cast<__nv_bfloat16*>(r.k_cache)[coff[j] + head_off] = __float2bfloat16_rn(y);
        }
      }
    }
    return;
  }
  const int n = tile * BM + row;
  if (n >= a.n) return;
  float v[NT];
#pragma unroll
  for (int m = 0; m < NT; ++m) v[m] = acc[m];
  if (MODE == kGemmResidual) {
    // Every residual load before the first store: y may be the residual itself (in place), so a store could
    // not be moved past a later load, and interleaving them would serialise the loads' latencies.
    __nv_bfloat16 r[NT];
#pragma unroll
    for (int m = 0; m < NT; ++m) r[m] = m < a.rows ? a.residual[(int64_t)m * a.ld_res + n] : __float2bfloat16_rn(0.f);
#pragma unroll
    for (int m = 0; m < NT; ++m) v[m] += __bfloat162float(r[m]);
  }
#pragma unroll
  for (int m = 0; m < NT; ++m)
    if (m < a.rows) a.y[(int64_t)m * a.ld_y + n] = __float2bfloat16_rn(v[m]);
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
  const int64_t total = (int64_t)a.tiles * a.chunks;
  const int64_t u0 = (int64_t)blockIdx.x * a.per;
  const int64_t u1 = min(total, u0 + a.per);
  if (u0 >= u1) return;  // uniform over the CTA

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
  grid_dependency_wait();  // the tokens come from the kernel before (launched as a programmatic dependent)
  const uint32_t tbase = tmem_base;
  const int first_tile = (int)(u0 / a.chunks);

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int i = 0;
      for (int64_t u = u0; u < u1 && !abort_flag; ++u, ++i) {
        const int t = (int)(u / a.chunks), c = (int)(u % a.chunks);
        const int s = i % STAGES, use = i / STAGES;
        if (use >= 1 && !mbar_wait(&empty[s], (use - 1) & 1)) {
          abort_flag = 1;
          break;
        }
        unsigned char* st = smem + s * L::STAGE;
        mbar_arrive_expect_tx(&full[s], L::STAGE);
#pragma unroll
        for (int j = 0; j < KB; ++j) {  // the weight boxes back to back: each row's KB * 128 bytes together
          const int kx = c * BKU + j * BK;
          if (MODE == kGemmSwiglu) {
            tma_load_2d(st + j * W_BOX, &wmap, kx, t * 64, &full[s]);                   // gate rows
            tma_load_2d(st + j * W_BOX + W_BOX / 2, &wmap, kx, a.n + t * 64, &full[s]);  // inner rows
          } else {
            tma_load_2d(st + j * W_BOX, &wmap, kx, t * BM, &full[s]);
          }
        }
#pragma unroll
        for (int j = 0; j < KB; ++j) tma_load_2d(st + W_BYTES + j * L::X_BOX, &xmap, c * BKU + j * BK, 0, &full[s]);
        issued = i + 1;
      }
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
      if (!mbar_wait(&acc_full[buf], (seg >> 1) & 1)) abort_flag = 1;
      tc_fence_after();
      __syncwarp();
      float acc[NT];
#pragma unroll
      for (int c = 0; c < NT; c += 16) tmem_ld16(tbase + lane_off + buf * NT + c, acc + c);
      tc_fence_before();
      mbar_arrive(&acc_free[buf]);
      if (whole) {
        finish_tile<NT, MODE>(a, t, row, acc, xch, 1);
      } else {
        const int slot = t == first_tile ? 0 : 1;
        float* dst = a.part + (((int64_t)blockIdx.x * 2 + slot) * BM + row) * NT;
#pragma unroll
        for (int m = 0; m < NT; m += 4) *reinterpret_cast<float4*>(dst + m) = make_float4(acc[m], acc[m + 1], acc[m + 2], acc[m + 3]);
        // Arrive on the tile's counter; the last CTA to arrive sums every covering CTA's partial and finishes it.
        __threadfence();
        named_sync(2, 128);
        const int64_t c0 = (int64_t)t * a.chunks;
        const int b0 = (int)(c0 / a.per), b1 = (int)((c0 + a.chunks - 1) / a.per);
        if (row == 0) *last_flag = atomicAdd(&a.counters[t], 1) == b1 - b0;
        named_sync(2, 128);
        if (*last_flag) {
          __threadfence();
          float sum[NT];
#pragma unroll
          for (int m = 0; m < NT; ++m) sum[m] = 0.f;
          for (int b = b0; b <= b1; ++b) {
            const int sl = t == (int)(((int64_t)b * a.per) / a.chunks) ? 0 : 1;
            const float4* src = reinterpret_cast<const float4*>(a.part + (((int64_t)b * 2 + sl) * BM + row) * NT);
#pragma unroll
            for (int m = 0; m < NT; m += 4) {
              const float4 v = __ldcg(src + m / 4);  // other CTAs' stores: from L2, not a stale L1 line
              sum[m] += v.x;
              sum[m + 1] += v.y;
              sum[m + 2] += v.z;
              sum[m + 3] += v.w;
            }
          }
          finish_tile<NT, MODE>(a, t, row, sum, xch, 1);
          if (row == 0) a.counters[t] = 0;  // zero again for the next call
        }
      }
      u = seg_end;
      if (abort_flag) break;
    }
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
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, L::TMEM_COLS);
  }
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
  return launch_dependent(wgemm_kernel<NT, MODE>, dim3((unsigned)a.grid), dim3(THREADS), (size_t)L::BYTES, stream, wm,
                          xm, a);
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
  int grid = device_sm_count();
  if (grid > total) grid = (int)total;
  a.per = (total + grid - 1) / grid;
  a.grid = (int)((total + a.per - 1) / a.per);
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
