// Split-KV attention over a KV cache: plan, partial-result layout and internal launchers.
//
// A "group" is a set of `nq` query rows that share one cache row's keys:
//   * decode (q_len 1):          group = batch row, nq = 1
//   * draft verify (q_len 1+k):  group = batch row, nq = 1+k, causal (query i sees lengths[g] + i keys)
//   * beam context:              group = input, nq = beams (every beam sees ctx_len[g] keys)
//   * beam generated part:       group = beam row, nq = 1, key j read from cache row ptr[r, j]
// Each CTA handles one (group, head, key split, query block); it writes an unnormalised partial
// output and its (max, sum) statistics, and a combine kernel merges the splits.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

namespace omni {

enum DType : int { kBF16 = 0, kF32 = 1 };

struct SplitArgs {
  const void* q;  // [rows_q, heads, D], contiguous; row of query i of group g = g * nq + i
  const void* k;  // cache [cache_rows, heads, cache_len, D] with strides s_kb, s_kh, s_ks (elements)
  const void* v;  // same strides as k
  int64_t s_kb, s_kh, s_ks;
  int64_t cache_rows, cache_len;
  const int64_t* lengths;  // [groups]
  const int32_t* ptr;      // gather mode only: [groups, ptr_stride] source cache row of key j
  int64_t ptr_stride;
  float* part_o;          // [rows_q, heads, st, D]
  float* part_ml;         // [rows_q, heads, st, 2] (max in log2 units, sum)
  int st;                 // splits held per (row, head) in the partial arrays
  int sp_offset;          // first split index written by this launch
  int heads, nq, causal, chunk, qblocks;
  int64_t key_bound;      // splits * chunk: keys the launch covers
  float qscale;           // softmax scale * log2(e)
  int* status;
};

struct SplitPlan {
  int nqb;      // queries per CTA (compile-time variant: 1, 2, 4 or 8)
  int qblocks;  // CTAs per group along the queries
  int splits;   // key splits
  int chunk;    // keys per split (a multiple of the tile)
};

// Key-split plan for `units` (group, head) pairs over `keys` keys.
SplitPlan plan_split(int dtype, int dim, int groups, int heads, int nq, int64_t keys);

// Bytes of the partial arrays for rows_q query rows with st splits each.
size_t partial_bytes(int64_t rows_q, int heads, int st, int dim);
void carve_partials(void* ws, int64_t rows_q, int heads, int st, int dim, float** part_o, float** part_ml);

cudaError_t launch_split(int dtype, int dim, bool gather, const SplitPlan& plan, const SplitArgs& a, int groups,
                         cudaStream_t stream);
cudaError_t launch_combine(int dtype, int dim, const float* part_o, const float* part_ml, void* out,
                           int64_t rows_heads, int st, cudaStream_t stream);

// Tensor-core pass (bf16, head_dim 128 or 512, 1..16 queries per group): persistent stream-K split, see
// attention_tc.cu.
struct TcParams {
  const __nv_bfloat16* q;  // [groups * nq, heads, dim]
  const int64_t* lengths;  // [groups]
  int groups, nq, causal, heads;
  int dim;        // head_dim: 128 or 512
  int kv_div;     // groups per cache row: group g reads cache row g / kv_div (1 but in prefill mode)
  int prefill;    // prefill mode: lengths[g] = (g % kv_div) * nq + 1, partials indexed by the unit's first CTA
  int64_t cap;    // min(cache length, keys): keys a unit may read (set by launch_tc_pass)
  float qscale;   // softmax scale * log2(e)
  float* part_o;  // [groups * nq, heads, st, dim]
  float* part_ml; // [groups * nq, heads, st, 2]
  int st;         // segments per (row, head) (set by launch_tc_pass)
  int grid;       // CTAs of the pass (set by launch_tc_pass)
  int unit_cost;  // scheduling cost of a unit's start, in eighths of a tile (set by launch_tc_pass)
  int prefetch;   // tiles prefetched into L2 ahead of the loads (set by launch_tc_pass)
  __nv_bfloat16* out;  // [groups * nq, heads, dim]: units a single CTA finishes are written here directly
                       // (null: every unit goes through the combine, e.g. when a second pass adds partials)
  unsigned* counters;  // [groups * heads] segments published per unit, zero on entry and left zero; non-null (with
                       // out): the last CTA to finish a unit merges its segments itself and no combine runs
  int* status;
};

// Decode / draft workspaces start with kCounterBytes of unit counters (zero before the first call, left zero by
// every call), then the split partials. Shapes with more than kCounterUnits (group, head) units merge in a combine.
constexpr int kCounterUnits = 16384;
constexpr size_t kCounterBytes = kCounterUnits * sizeof(unsigned);

bool tc_path_enabled(int dtype, int dim, int nq);
int tc_segments(int64_t keys);
int tc_grid();
int tc_unit_cost(int nq);
// Prefill mode of the pass: the segments a unit can span (the partial slots per CTA) for batch rows of `width`
// queries in groups of `nq`, and the workspace bytes (unit counters, then the compact partials).
int tc_prefill_segments(int batch, int heads, int width, int nq);
size_t tc_prefill_workspace(int batch, int heads, int width, int dim, int nq);
cudaError_t launch_tc_pass(const void* k, const void* v, int64_t cache_rows, int64_t cache_len, int64_t s_row,
                           int64_t s_head, int64_t s_pos, int keys, TcParams& p, cudaStream_t stream);
// Beam search's generated keys, attended inside the combine (before it waits for the pass): row r's key j < gen_len[r]
// comes from cache row ptr[r, j] at position j (bf16, head_dim as the pass's).
struct GenKeys {
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t s_kb, s_kh, s_ks, cache_rows, cache_len;  // strides in elements
  const int32_t* ptr;
  int64_t ptr_stride;
  const int64_t* gen_len;  // [rows]
  int enabled;
};

// Merges the pass's segments (and, for beam search, the generated keys' attention) into out.
cudaError_t launch_tc_combine(const TcParams& p, void* out, const GenKeys& gen, cudaStream_t stream);

bool dim_supported(int dtype, int dim);
int device_sm_count();

}  // namespace omni
