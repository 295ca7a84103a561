// Split-KV flash-decode attention on CUDA cores (every dtype / head_dim / query count), and the
// split-combine.
//
// Work of one CTA: a (group, head, key split, query block). Keys and values of the split stream
// through a 4-stage shared-memory ring filled by 1-D bulk copies (TMA engine) on mbarriers, so
// the loads of the next tiles are in flight while a tile is consumed. 256 threads form "teams"
// of L lanes; a team owns one key at a time, each lane a 16-byte slice of it, and keeps its own
// online-softmax state (max, sum, output slice) per query, so no cross-team synchronisation is
// needed inside the key loop. The teams' states are merged once at the end of the split.
//
// Algorithm of the reference this restates: omniasr_trt/kernels.py:163-211 (_attn_split /
// _attn_combine), kernels.py:56-161 (_beam_ctx / _beam_gen / _beam_combine).

#include <math.h>
#include <stdlib.h>

#include "attention.cuh"
#include "common.cuh"

namespace omni {

template <typename T, int D>
struct SplitShape {
  static constexpr int kVec = Elem<T>::kVec;
  static constexpr int kRowBytes = D * (int)sizeof(T);
  static constexpr int kChunks = D / kVec;  // 16-byte chunks per key row
  static constexpr int kLanes = kChunks < 32 ? kChunks : 32;
  static constexpr int kCpl = kChunks / kLanes;  // chunks per lane
  static constexpr int kEpt = kCpl * kVec;       // elements per lane
  static constexpr int kThreads = 256;
  static constexpr int kSlots = kThreads / kLanes;  // teams (keys processed side by side)
  static constexpr int kTileRaw = 8192 / kRowBytes;
  static constexpr int kTile = kTileRaw > kSlots ? kTileRaw : kSlots;  // keys per ring stage
  static constexpr int kStages = 4;
  static constexpr int kRingBytes = kStages * 2 * kTile * kRowBytes;
  static constexpr int kMergeBytes = kSlots * (D + 2) * 4;
  static constexpr int kSmemBytes = kRingBytes > kMergeBytes ? kRingBytes : kMergeBytes;
  static_assert(kChunks % kLanes == 0, "head_dim");
  static_assert(kTile % kSlots == 0, "tile");
};

template <typename T, int D, int NQB, bool GATHER>
__global__ void __launch_bounds__(256) split_attention_kernel(const SplitArgs a) {
  using S = SplitShape<T, D>;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t full[S::kStages];
  __shared__ volatile int abort_flag;

  const int tid = threadIdx.x;
  const int team = tid / S::kLanes;
  const int lane = tid % S::kLanes;
  const int warp = tid >> 5;
  const int wlane = tid & 31;
  const int g = blockIdx.x / a.qblocks;
  const int q0 = (blockIdx.x % a.qblocks) * NQB;
  const int h = blockIdx.y;
  const int sp = blockIdx.z;
  const int nqb = min(NQB, a.nq - q0);

  // Keys seen by each query of the block, clamped to the cache (a clamp is an index error).
  int64_t n = a.lengths[g];
  bool bad = n < 0;
  int64_t lim[NQB];
  int64_t need = 0;
#pragma unroll
  for (int i = 0; i < NQB; ++i) {
    int64_t li = a.causal ? n + q0 + i : n;
    if (i < nqb && (li > a.cache_len || li > a.key_bound)) bad = true;
    li = li < 0 ? 0 : li;
    li = li > a.cache_len ? a.cache_len : li;
    lim[i] = li;
    if (i < nqb && li > need) need = li;
  }
  if (bad && tid == 0 && sp == 0) raise_status(a.status, kStatusIndex);

  const int64_t start = (int64_t)sp * a.chunk;
  const int64_t stop = min(start + (int64_t)a.chunk, need);
  const int64_t row0 = (int64_t)g * a.nq + q0;  // query row of the block's first query
  const int64_t qstride = (int64_t)a.heads * a.st;  // partial entries between consecutive query rows
  const int64_t part0 = (row0 * a.heads + h) * a.st + a.sp_offset + sp;
  if (stop <= start) {  // nothing to read: an empty split (the combine skips it)
    if (tid < nqb) reinterpret_cast<float2*>(a.part_ml)[part0 + tid * qstride] = make_float2(-INFINITY, 0.f);
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < S::kStages; ++s) mbar_init(&full[s], 1);
    mbar_fence_init();
    abort_flag = 0;
  }

  // This lane's slice of each query, pre-scaled so that scores come out in log2 units.
  float qf[NQB][S::kEpt];
  {
    const T* qb = reinterpret_cast<const T*>(a.q) + (row0 * a.heads + h) * D;
#pragma unroll
    for (int i = 0; i < NQB; ++i) {
#pragma unroll
      for (int c = 0; c < S::kCpl; ++c) {
        float f[S::kVec];
        if (i < nqb) {
          const uint4 u = __ldg(reinterpret_cast<const uint4*>(qb + (int64_t)i * a.heads * D) + lane + c * S::kLanes);
          Elem<T>::unpack(u, f);
        } else {
#pragma unroll
          for (int e = 0; e < S::kVec; ++e) f[e] = 0.f;
        }
#pragma unroll
        for (int e = 0; e < S::kVec; ++e) qf[i][c * S::kVec + e] = f[e] * a.qscale;
      }
    }
  }
  __syncthreads();

  const char* kbase = reinterpret_cast<const char*>(a.k);
  const char* vbase = reinterpret_cast<const char*>(a.v);
  const int64_t head_off = (int64_t)h * a.s_kh;
  const int ntiles = (int)((stop - start + S::kTile - 1) / S::kTile);
  const bool contiguous = !GATHER && a.s_ks == D;

  // Tile t -> stage t % kStages (warp 0 only).
  auto issue = [&](int t) {
    const int stage = t % S::kStages;
    const int64_t k0 = start + (int64_t)t * S::kTile;
    const int nk = (int)min((int64_t)S::kTile, stop - k0);
    unsigned char* ks = smem + stage * 2 * S::kTile * S::kRowBytes;
    unsigned char* vs = ks + S::kTile * S::kRowBytes;
    if (wlane == 0) mbar_arrive_expect_tx(&full[stage], 2u * nk * S::kRowBytes);
    __syncwarp();
    if (contiguous) {
      if (wlane == 0) {
        const int64_t off = ((int64_t)g * a.s_kb + head_off + k0 * D) * (int64_t)sizeof(T);
        bulk_g2s(ks, kbase + off, nk * S::kRowBytes, &full[stage]);
        bulk_g2s(vs, vbase + off, nk * S::kRowBytes, &full[stage]);
      }
    } else {
      for (int j = wlane; j < nk; j += 32) {
        int64_t row = g;
        if (GATHER) {
          const int64_t src = a.ptr[(int64_t)g * a.ptr_stride + k0 + j];
          if (src < 0 || src >= a.cache_rows) {
            raise_status(a.status, kStatusIndex);
          } else {
            row = src;
          }
        }
        const int64_t off = (row * a.s_kb + head_off + (k0 + j) * a.s_ks) * (int64_t)sizeof(T);
        bulk_g2s(ks + j * S::kRowBytes, kbase + off, S::kRowBytes, &full[stage]);
        bulk_g2s(vs + j * S::kRowBytes, vbase + off, S::kRowBytes, &full[stage]);
      }
    }
  };

  if (warp == 0) {
    for (int t = 0; t < S::kStages && t < ntiles; ++t) issue(t);
  }

  float m[NQB], l[NQB], acc[NQB][S::kEpt];
#pragma unroll
  for (int i = 0; i < NQB; ++i) {
    m[i] = -INFINITY;
    l[i] = 0.f;
#pragma unroll
    for (int e = 0; e < S::kEpt; ++e) acc[i][e] = 0.f;
  }

  int t = 0;
  for (; t < ntiles; ++t) {
    const int stage = t % S::kStages;
    if (!mbar_wait(&full[stage], (t / S::kStages) & 1)) abort_flag = 1;
    const int64_t k0 = start + (int64_t)t * S::kTile;
    const int nk = (int)min((int64_t)S::kTile, stop - k0);
    const unsigned char* ks = smem + stage * 2 * S::kTile * S::kRowBytes;
    const unsigned char* vs = ks + S::kTile * S::kRowBytes;
#pragma unroll
    for (int u = 0; u < S::kTile / S::kSlots; ++u) {
      const int j = team + u * S::kSlots;
      const bool valid = j < nk;
      const int64_t key = k0 + j;
      float kf[S::kEpt];
#pragma unroll
      for (int c = 0; c < S::kCpl; ++c)
        Elem<T>::unpack(*reinterpret_cast<const uint4*>(ks + j * S::kRowBytes + (lane + c * S::kLanes) * 16),
                        kf + c * S::kVec);
      float dot[NQB];
#pragma unroll
      for (int i = 0; i < NQB; ++i) {
        float d0 = 0.f;
#pragma unroll
        for (int e = 0; e < S::kEpt; ++e) d0 = fmaf(qf[i][e], kf[e], d0);
        dot[i] = d0;
      }
#pragma unroll
      for (int i = 0; i < NQB; ++i) {
#pragma unroll
        for (int o = S::kLanes / 2; o > 0; o >>= 1) dot[i] += __shfl_xor_sync(0xffffffffu, dot[i], o);
      }
      float vf[S::kEpt];
#pragma unroll
      for (int c = 0; c < S::kCpl; ++c)
        Elem<T>::unpack(*reinterpret_cast<const uint4*>(vs + j * S::kRowBytes + (lane + c * S::kLanes) * 16),
                        vf + c * S::kVec);
#pragma unroll
      for (int i = 0; i < NQB; ++i) {
        if (valid && i < nqb && key < lim[i]) {
          const float mn = fmaxf(m[i], dot[i]);
          const float corr = ex2(m[i] - mn);
          const float p = ex2(dot[i] - mn);
          l[i] = fmaf(l[i], corr, p);
#pragma unroll
          for (int e = 0; e < S::kEpt; ++e) acc[i][e] = fmaf(acc[i][e], corr, p * vf[e]);
          m[i] = mn;
        }
      }
    }
    __syncthreads();
    if (abort_flag) break;
    if (warp == 0 && t + S::kStages < ntiles) issue(t + S::kStages);
  }

  if (abort_flag) {
    // A wait gave up: record it, let the copies already issued land (bounded), and stop.
    if (tid == 0) {
      raise_status(a.status, kStatusTimeout);
      for (int u = t; u < ntiles && u < t + S::kStages; ++u) mbar_wait(&full[u % S::kStages], (u / S::kStages) & 1);
    }
    __syncthreads();
    return;
  }

  // Merge the teams' states of each query; the ring is free now.
  float* red = reinterpret_cast<float*>(smem);
  float* po = a.part_o + part0 * D;
  for (int i = 0; i < nqb; ++i) {
    float mi = m[0], li = l[0];
#pragma unroll
    for (int u = 0; u < NQB; ++u)
      if (u == i) mi = m[u], li = l[u];
    float* mine = red + team * (D + 2);
#pragma unroll
    for (int u = 0; u < NQB; ++u) {
      if (u == i) {
#pragma unroll
        for (int c = 0; c < S::kCpl; ++c)
#pragma unroll
          for (int e = 0; e < S::kVec; ++e) mine[(lane + c * S::kLanes) * S::kVec + e] = acc[u][c * S::kVec + e];
      }
    }
    if (lane == 0) {
      mine[D] = mi;
      mine[D + 1] = li;
    }
    __syncthreads();
    float mx = -INFINITY;
    for (int s = 0; s < S::kSlots; ++s) mx = fmaxf(mx, red[s * (D + 2) + D]);
    for (int d = tid; d < D; d += S::kThreads) {
      float o = 0.f, lsum = 0.f;
      if (mx != -INFINITY) {
        for (int s = 0; s < S::kSlots; ++s) {
          const float ms = red[s * (D + 2) + D];
          if (ms != -INFINITY) {
            const float w = ex2(ms - mx);
            o = fmaf(w, red[s * (D + 2) + d], o);
            lsum = fmaf(w, red[s * (D + 2) + D + 1], lsum);
          }
        }
      }
      po[i * qstride * D + d] = o;
      if (d == 0) reinterpret_cast<float2*>(a.part_ml)[part0 + i * qstride] = make_float2(mx, lsum);
    }
    __syncthreads();
  }
}

// out[r, h] = sum_s w_s o_s / sum_s w_s l_s with w_s = 2^(m_s - max); zeros when no split saw a key.
template <typename T, int D>
__global__ void __launch_bounds__(128) combine_kernel(const float* __restrict__ part_o,
                                                      const float* __restrict__ part_ml, T* __restrict__ out,
                                                      int st) {
  const int64_t rh = blockIdx.x;
  const float2* ml = reinterpret_cast<const float2*>(part_ml) + rh * st;
  float mx = -INFINITY;
  for (int s = 0; s < st; ++s) mx = fmaxf(mx, ml[s].x);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f, lsum = 0.f;
    if (mx != -INFINITY) {
      for (int s = 0; s < st; ++s) {
        const float2 e = ml[s];
        if (e.x != -INFINITY) {
          const float w = ex2(e.x - mx);
          o = fmaf(w, part_o[(rh * st + s) * D + d], o);
          lsum = fmaf(w, e.y, lsum);
        }
      }
    }
    out[rh * D + d] = Elem<T>::from_float(lsum > 0.f ? o / lsum : o);
  }
}

// ---------------------------------------------------------------------------------------------
// Host side.

namespace {

template <typename T, int D>
int tile_keys() {
  return SplitShape<T, D>::kTile;
}

int tile_for(int dtype, int dim) {
#define OMNI_TILE(DD) \
  case DD:            \
    return dtype == kBF16 ? tile_keys<__nv_bfloat16, DD>() : tile_keys<float, DD>();
  switch (dim) {
    OMNI_TILE(16)
    OMNI_TILE(32)
    OMNI_TILE(64)
    OMNI_TILE(128)
    OMNI_TILE(256)
    OMNI_TILE(512)
  }
#undef OMNI_TILE
  return 0;
}

int split_target_ctas() {
  static int target = [] {
    const char* e = getenv("OMNIASR_SPLIT_CTAS_PER_SM");
    const int per_sm = e ? atoi(e) : 4;
    return device_sm_count() * (per_sm > 0 ? per_sm : 4);
  }();
  return target;
}

template <typename T, int D, int NQB, bool GATHER>
cudaError_t launch_split_t(const SplitPlan& p, const SplitArgs& a, int groups, cudaStream_t stream) {
  using S = SplitShape<T, D>;
  auto kern = split_attention_kernel<T, D, NQB, GATHER>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, S::kSmemBytes);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  dim3 grid((unsigned)(groups * p.qblocks), (unsigned)a.heads, (unsigned)p.splits);
  kern<<<grid, S::kThreads, S::kSmemBytes, stream>>>(a);
  return cudaGetLastError();
}

template <typename T, int D>
cudaError_t launch_split_d(bool gather, const SplitPlan& p, const SplitArgs& a, int groups, cudaStream_t s) {
  if (gather) return launch_split_t<T, D, 1, true>(p, a, groups, s);
  switch (p.nqb) {
    case 1:
      return launch_split_t<T, D, 1, false>(p, a, groups, s);
    case 2:
      return launch_split_t<T, D, 2, false>(p, a, groups, s);
    case 4:
      return launch_split_t<T, D, 4, false>(p, a, groups, s);
    default:
      return launch_split_t<T, D, 8, false>(p, a, groups, s);
  }
}

template <typename T>
cudaError_t launch_split_dt(int dim, bool gather, const SplitPlan& p, const SplitArgs& a, int groups,
                            cudaStream_t s) {
  switch (dim) {
    case 16:
      return launch_split_d<T, 16>(gather, p, a, groups, s);
    case 32:
      return launch_split_d<T, 32>(gather, p, a, groups, s);
    case 64:
      return launch_split_d<T, 64>(gather, p, a, groups, s);
    case 128:
      return launch_split_d<T, 128>(gather, p, a, groups, s);
    case 256:
      return launch_split_d<T, 256>(gather, p, a, groups, s);
    case 512:
      return launch_split_d<T, 512>(gather, p, a, groups, s);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t launch_combine_t(int dim, const float* po, const float* pml, void* out, int64_t rh, int st,
                             cudaStream_t s) {
  const unsigned threads = dim < 128 ? (unsigned)dim : 128u;
  T* o = reinterpret_cast<T*>(out);
  switch (dim) {
    case 16:
      combine_kernel<T, 16><<<(unsigned)rh, threads, 0, s>>>(po, pml, o, st);
      break;
    case 32:
      combine_kernel<T, 32><<<(unsigned)rh, threads, 0, s>>>(po, pml, o, st);
      break;
    case 64:
      combine_kernel<T, 64><<<(unsigned)rh, threads, 0, s>>>(po, pml, o, st);
      break;
    case 128:
      combine_kernel<T, 128><<<(unsigned)rh, threads, 0, s>>>(po, pml, o, st);
      break;
    case 256:
      combine_kernel<T, 256><<<(unsigned)rh, threads, 0, s>>>(po, pml, o, st);
      break;
    case 512:
      combine_kernel<T, 512><<<(unsigned)rh, threads, 0, s>>>(po, pml, o, st);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace

bool dim_supported(int dtype, int dim) {
  return (dtype == kBF16 || dtype == kF32) &&
         (dim == 16 || dim == 32 || dim == 64 || dim == 128 || dim == 256 || dim == 512);
}

int device_sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  return n;
}

SplitPlan plan_split(int dtype, int dim, int groups, int heads, int nq, int64_t keys) {
  SplitPlan p;
  p.nqb = nq <= 1 ? 1 : nq <= 2 ? 2 : nq <= 4 ? 4 : 8;
  p.qblocks = (nq + p.nqb - 1) / p.nqb;
  const int tile = tile_for(dtype, dim);
  const int64_t min_chunk = tile * ((128 + tile - 1) / tile);  // >= 128 keys per split
  const int64_t units = (int64_t)groups * heads * p.qblocks;
  int64_t want = units > 0 ? (split_target_ctas() + units - 1) / units : 1;
  int64_t most = (keys + min_chunk - 1) / min_chunk;
  int64_t splits = want < most ? want : most;
  if (splits < 1) splits = 1;
  int64_t chunk = (keys + splits - 1) / splits;
  chunk = (chunk + tile - 1) / tile * tile;
  if (chunk < tile) chunk = tile;
  splits = (keys + chunk - 1) / chunk;
  if (splits < 1) splits = 1;
  p.splits = (int)splits;
  p.chunk = (int)chunk;
  return p;
}

size_t partial_bytes(int64_t rows_q, int heads, int st, int dim) {
  const size_t ml = (size_t)rows_q * heads * st * 2 * sizeof(float);
  const size_t ml_aligned = (ml + 255) / 256 * 256;
  return ml_aligned + (size_t)rows_q * heads * st * dim * sizeof(float);
}

void carve_partials(void* ws, int64_t rows_q, int heads, int st, int dim, float** part_o, float** part_ml) {
  const size_t ml = (size_t)rows_q * heads * st * 2 * sizeof(float);
  const size_t ml_aligned = (ml + 255) / 256 * 256;
  *part_ml = reinterpret_cast<float*>(ws);
  *part_o = reinterpret_cast<float*>(reinterpret_cast<char*>(ws) + ml_aligned);
}

cudaError_t launch_split(int dtype, int dim, bool gather, const SplitPlan& plan, const SplitArgs& a, int groups,
                         cudaStream_t stream) {
  if (groups <= 0 || a.heads <= 0) return cudaSuccess;
  if (dtype == kBF16) return launch_split_dt<__nv_bfloat16>(dim, gather, plan, a, groups, stream);
  return launch_split_dt<float>(dim, gather, plan, a, groups, stream);
}

cudaError_t launch_combine(int dtype, int dim, const float* part_o, const float* part_ml, void* out,
                           int64_t rows_heads, int st, cudaStream_t stream) {
  if (rows_heads <= 0) return cudaSuccess;
  if (dtype == kBF16) return launch_combine_t<__nv_bfloat16>(dim, part_o, part_ml, out, rows_heads, st, stream);
  return launch_combine_t<float>(dim, part_o, part_ml, out, rows_heads, st, stream);
}

}  // namespace omni
