// extern "C" entry points (include/omniasr_b200.h): argument checks, split plans, launches.

#include <math.h>
#include <stdarg.h>
#include <stdio.h>

#include <string>

#include "attention.cuh"
#include "beam.cuh"
#include "gather.cuh"
#include "omniasr_b200.h"
#include "prefill.cuh"
#include "rope_kv.cuh"
#include "spec.cuh"
#include "wgemm.cuh"

static_assert(omni::kCounterBytes == OMNIASR_ATTENTION_COUNTER_BYTES, "counter prefix of the decode / draft workspace");

// Query positions per group of the grouped prefill: the tensor-core pass's widest unit.
constexpr int kPrefillGroup = 16;

namespace {

thread_local std::string g_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_error = buf;
  return code;
}

int ok() {
  g_error.clear();
  return OMNIASR_OK;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(OMNIASR_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return ok();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int esize(int dtype) { return dtype == OMNIASR_BF16 ? 2 : 4; }

bool stride_ok(int64_t stride, int dtype) { return stride >= 0 && (stride * esize(dtype)) % 16 == 0; }

int check_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(OMNIASR_ERR_DEVICE, "no CUDA device");
  if (!omniasr_device_supported(dev))
    return fail(OMNIASR_ERR_DEVICE, "device %d is not compute capability 10.0 (sm_100a code)", dev);
  return OMNIASR_OK;
}

int check_common(int dtype, int dim, int heads) {
  if (dtype != OMNIASR_BF16 && dtype != OMNIASR_F32) return fail(OMNIASR_ERR_UNSUPPORTED, "dtype %d", dtype);
  if (!omni::dim_supported(dtype, dim))
    return fail(OMNIASR_ERR_UNSUPPORTED, "head_dim %d (supported: 16, 32, 64, 128, 256, 512)", dim);
  if (heads <= 0 || heads > 65535) return fail(OMNIASR_ERR_ARGUMENT, "heads %d", heads);
  return check_device();
}

int check_cache(const char* name, const void* k, const void* v, int64_t rows, int64_t len, int64_t s_row,
                int64_t s_head, int64_t s_pos, int heads, int dim, int dtype) {
  if (!k || !v) return fail(OMNIASR_ERR_ARGUMENT, "%s: null cache pointer", name);
  if (!aligned16(k) || !aligned16(v)) return fail(OMNIASR_ERR_ARGUMENT, "%s: cache not 16-byte aligned", name);
  if (!stride_ok(s_row, dtype) || !stride_ok(s_head, dtype) || !stride_ok(s_pos, dtype))
    return fail(OMNIASR_ERR_ARGUMENT, "%s: cache strides (%lld, %lld, %lld) must keep 16-byte alignment", name,
                (long long)s_row, (long long)s_head, (long long)s_pos);
  if (rows < 0 || len < 0) return fail(OMNIASR_ERR_ARGUMENT, "%s: cache extents", name);
  if (s_pos < dim && len > 1) return fail(OMNIASR_ERR_ARGUMENT, "%s: positions overlap (stride %lld < dim %d)", name,
                                          (long long)s_pos, dim);
  (void)heads;
  return OMNIASR_OK;
}

}  // namespace

namespace omni {
// Sets this thread's last-error message (for entry points defined in other files); returns `code`.
int set_last_error(int code, const char* message) { return fail(code, "%s", message); }
}  // namespace omni

extern "C" {

int omniasr_abi_version(void) { return 2; }

const char* omniasr_last_error(void) { return g_error.c_str(); }

int omniasr_device_supported(int device) {
  static int cache[64] = {0};  // 0 unknown, 1 yes, 2 no
  if (device < 0) return 0;
  if (device < 64 && cache[device]) return cache[device] == 1;
  int major = 0, minor = 0;
  int ok_ = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) == cudaSuccess &&
            cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) == cudaSuccess &&
            major == 10 && minor == 0;
  if (device < 64) cache[device] = ok_ ? 1 : 2;
  return ok_;
}

int omniasr_splits_for(int rows, int heads, int keys, int block, int programs, int* splits, int* chunk) {
  if (rows <= 0 || heads <= 0 || block <= 0 || !splits || !chunk)
    return fail(OMNIASR_ERR_ARGUMENT, "splits_for: rows %d heads %d block %d", rows, heads, block);
  int want = programs / (rows * heads);
  if (want < 1) want = 1;
  int s = 1;
  while (s * 2 <= want && (int64_t)s * 2 * block <= keys) s *= 2;
  const int c = (keys + s - 1) / s;
  *splits = s;
  *chunk = (c + block - 1) / block * block;
  return ok();
}

size_t omniasr_attention_workspace(int kind, int dtype, int groups, int per_group, int heads, int dim, int64_t keys,
                                   int64_t gen_keys) {
  if (groups <= 0 || per_group <= 0 || heads <= 0 || !omni::dim_supported(dtype, dim)) return 0;
  const int64_t rows_q = (int64_t)groups * per_group;
  const int nq = kind == OMNIASR_DECODE ? 1 : per_group;
  if (kind == OMNIASR_BEAM) {
    const omni::SplitPlan g = omni::plan_split(dtype, dim, (int)rows_q, heads, 1, gen_keys);
    if (omni::tc_path_enabled(dtype, dim, nq))
      return omni::partial_bytes(rows_q, heads, omni::tc_segments(keys), dim) +
             omni::partial_bytes(rows_q, heads, g.splits, dim);
    const omni::SplitPlan c = omni::plan_split(dtype, dim, groups, heads, per_group, keys);
    return omni::partial_bytes(rows_q, heads, c.splits + g.splits, dim);
  }
  // Decode and draft workspaces: the unit counters, then the partials.
  if (omni::tc_path_enabled(dtype, dim, nq))
    return omni::kCounterBytes + omni::partial_bytes(rows_q, heads, omni::tc_segments(keys), dim);
  const omni::SplitPlan p = omni::plan_split(dtype, dim, groups, heads, nq, keys);
  return omni::kCounterBytes + omni::partial_bytes(rows_q, heads, p.splits, dim);
}

int omniasr_rope_kv(const void* qkv, int64_t qkv_stride, const float* cs, int64_t cs_positions, const int64_t* pos,
                    const int64_t* slots, const int64_t* cache_pos, void* q_out, void* k_cache, void* v_cache,
                    int64_t cache_rows, int64_t cache_len, int64_t stride_row, int64_t stride_head,
                    int64_t stride_pos, int n, int heads, int dim, int dtype, int* status, cudaStream_t stream) {
  if (int e = check_common(dtype, dim, heads)) return e;
  if (n < 0) return fail(OMNIASR_ERR_ARGUMENT, "rope_kv: n %d", n);
  if (n == 0) return ok();
  if (!qkv || !cs || !pos || !q_out) return fail(OMNIASR_ERR_ARGUMENT, "rope_kv: null pointer");
  if (!aligned16(qkv) || !aligned16(cs) || !aligned16(q_out) || !stride_ok(qkv_stride, dtype))
    return fail(OMNIASR_ERR_ARGUMENT, "rope_kv: qkv / cs / q_out must be 16-byte aligned");
  if (qkv_stride < 3LL * heads * dim) return fail(OMNIASR_ERR_ARGUMENT, "rope_kv: qkv row stride %lld < 3*H*D",
                                                  (long long)qkv_stride);
  if (int e = check_cache("rope_kv", k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head, stride_pos,
                          heads, dim, dtype))
    return e;
  omni::RopeArgs a;
  a.qkv = qkv;
  a.qkv_stride = qkv_stride;
  a.cs = cs;
  a.cs_positions = cs_positions;
  a.pos = pos;
  a.slots = slots;
  a.cache_pos = cache_pos;
  a.q_out = q_out;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.s_kb = stride_row;
  a.s_kh = stride_head;
  a.s_ks = stride_pos;
  a.cache_rows = cache_rows;
  a.cache_len = cache_len;
  a.heads = heads;
  a.status = status;
  return cuda_status(omni::launch_rope_kv(dtype, dim, a, n, stream), "rope_kv launch");
}

}  // extern "C"

namespace omni {
// The argument checks of a decode / draft call, everything but the workspace: OMNIASR_OK or the error code (with
// the message set). groups == 0 passes (nothing to launch).
int check_group_args(const char* name, const void* q, const void* k_cache, const void* v_cache, int64_t cache_rows,
                     int64_t cache_len, int64_t stride_row, int64_t stride_head, int64_t stride_pos,
                     const int64_t* lengths, const void* out, int groups, int nq, int heads, int dim, int keys,
                     int dtype) {
  if (int e = check_common(dtype, dim, heads)) return e;
  if (groups < 0 || nq <= 0) return fail(OMNIASR_ERR_ARGUMENT, "%s: batch %d tokens %d", name, groups, nq);
  if (groups == 0) return ok();
  if (!q || !out || !lengths) return fail(OMNIASR_ERR_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(q) || !aligned16(out)) return fail(OMNIASR_ERR_ARGUMENT, "%s: q / out not 16-byte aligned", name);
  if (int e = check_cache(name, k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head, stride_pos, heads,
                          dim, dtype))
    return e;
  if (groups > cache_rows) return fail(OMNIASR_ERR_ARGUMENT, "%s: %d rows but the cache has %lld", name, groups,
                                       (long long)cache_rows);
  if (keys < 0 || keys > cache_len)
    return fail(OMNIASR_ERR_ARGUMENT, "%s: keys %d outside [0, cache length %lld]", name, keys, (long long)cache_len);
  return OMNIASR_OK;
}
}  // namespace omni

extern "C" {

static int group_attention(const char* name, const void* q, const void* k_cache, const void* v_cache,
                           int64_t cache_rows, int64_t cache_len, int64_t stride_row, int64_t stride_head,
                           int64_t stride_pos, const int64_t* lengths, void* out, int groups, int nq, int causal,
                           int heads, int dim, int keys, float scale, int dtype, void* workspace,
                           size_t workspace_bytes, int* status, cudaStream_t stream) {
  if (int e = omni::check_group_args(name, q, k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head,
                                     stride_pos, lengths, out, groups, nq, heads, dim, keys, dtype))
    return e;
  if (groups == 0) return ok();
  const int64_t rows_q = (int64_t)groups * nq;
  if (omni::tc_path_enabled(dtype, dim, nq)) {
    const size_t need = omni::kCounterBytes + omni::partial_bytes(rows_q, heads, omni::tc_segments(keys), dim);
    if (!workspace || workspace_bytes < need || !aligned16(workspace))
      return fail(OMNIASR_ERR_WORKSPACE, "%s: workspace %zu bytes, %zu needed (16-byte aligned)", name,
                  workspace ? workspace_bytes : (size_t)0, need);
    omni::TcParams t{};
    t.q = static_cast<const __nv_bfloat16*>(q);
    t.lengths = lengths;
    t.groups = groups;
    t.nq = nq;
    t.causal = causal;
    t.heads = heads;
    t.dim = dim;
    t.qscale = scale * omni::kLog2e;
    t.status = status;
    t.out = static_cast<__nv_bfloat16*>(out);
    // The last CTA to finish a unit merges its segments (no combine kernel) when the unit counters cover the shape.
    t.counters = (int64_t)groups * heads <= omni::kCounterUnits ? static_cast<unsigned*>(workspace) : nullptr;
    omni::carve_partials(static_cast<char*>(workspace) + omni::kCounterBytes, rows_q, heads, omni::tc_segments(keys),
                         dim, &t.part_o, &t.part_ml);
    if (int e = cuda_status(omni::launch_tc_pass(k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head,
                                                 stride_pos, keys, t, stream),
                            "tensor-core attention launch"))
      return e;
    if (t.counters) return ok();
    return cuda_status(omni::launch_tc_combine(t, out, omni::GenKeys{}, stream), "combine launch");
  }
  const omni::SplitPlan plan = omni::plan_split(dtype, dim, groups, heads, nq, keys);
  const size_t need = omni::kCounterBytes + omni::partial_bytes(rows_q, heads, plan.splits, dim);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return fail(OMNIASR_ERR_WORKSPACE, "%s: workspace %zu bytes, %zu needed (16-byte aligned)", name,
                workspace ? workspace_bytes : (size_t)0, need);
  float *po, *pml;
  omni::carve_partials(static_cast<char*>(workspace) + omni::kCounterBytes, rows_q, heads, plan.splits, dim, &po,
                       &pml);
  omni::SplitArgs a{};
  a.q = q;
  a.k = k_cache;
  a.v = v_cache;
  a.s_kb = stride_row;
  a.s_kh = stride_head;
  a.s_ks = stride_pos;
  a.cache_rows = cache_rows;
  a.cache_len = cache_len;
  a.lengths = lengths;
  a.part_o = po;
  a.part_ml = pml;
  a.st = plan.splits;
  a.sp_offset = 0;
  a.heads = heads;
  a.nq = nq;
  a.causal = causal;
  a.chunk = plan.chunk;
  a.qblocks = plan.qblocks;
  a.key_bound = (int64_t)plan.splits * plan.chunk;
  a.qscale = scale * omni::kLog2e;
  a.status = status;
  if (int e = cuda_status(omni::launch_split(dtype, dim, false, plan, a, groups, stream), "split launch")) return e;
  return cuda_status(omni::launch_combine(dtype, dim, po, pml, out, rows_q * heads, plan.splits, stream),
                     "combine launch");
}

int omniasr_decode_attention(const void* q, const void* k_cache, const void* v_cache, int64_t cache_rows,
                             int64_t cache_len, int64_t stride_row, int64_t stride_head, int64_t stride_pos,
                             const int64_t* lengths, void* out, int batch, int heads, int dim, int keys, float scale,
                             int dtype, void* workspace, size_t workspace_bytes, int* status, cudaStream_t stream) {
  return group_attention("decode_attention", q, k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head,
                         stride_pos, lengths, out, batch, 1, 0, heads, dim, keys, scale, dtype, workspace,
                         workspace_bytes, status, stream);
}

int omniasr_draft_attention(const void* q, const void* k_cache, const void* v_cache, int64_t cache_rows,
                            int64_t cache_len, int64_t stride_row, int64_t stride_head, int64_t stride_pos,
                            const int64_t* lengths, void* out, int batch, int tokens, int heads, int dim, int keys,
                            float scale, int dtype, void* workspace, size_t workspace_bytes, int* status,
                            cudaStream_t stream) {
  return group_attention("draft_attention", q, k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head,
                         stride_pos, lengths, out, batch, tokens, 1, heads, dim, keys, scale, dtype, workspace,
                         workspace_bytes, status, stream);
}

int omniasr_beam_attention(const void* q, const void* kc, const void* vc, int64_t ctx_rows, int64_t ctx_len_cap,
                           int64_t ctx_stride_row, int64_t ctx_stride_head, int64_t ctx_stride_pos,
                           const int64_t* ctx_len, const void* kg, const void* vg, int64_t gen_rows,
                           int64_t gen_len_cap, int64_t gen_stride_row, int64_t gen_stride_head,
                           int64_t gen_stride_pos, const int32_t* ptr, int64_t ptr_stride, const int64_t* gen_len,
                           void* out, int groups, int beams, int heads, int dim, int ctx_keys, float scale, int dtype,
                           void* workspace, size_t workspace_bytes, int* status, cudaStream_t stream) {
  const char* name = "beam_attention";
  if (int e = check_common(dtype, dim, heads)) return e;
  if (groups < 0 || beams <= 0) return fail(OMNIASR_ERR_ARGUMENT, "%s: groups %d beams %d", name, groups, beams);
  if (groups == 0) return ok();
  if (!q || !out || !ctx_len || !gen_len || !ptr) return fail(OMNIASR_ERR_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(q) || !aligned16(out)) return fail(OMNIASR_ERR_ARGUMENT, "%s: q / out not 16-byte aligned", name);
  if (int e = check_cache("beam_attention (context)", kc, vc, ctx_rows, ctx_len_cap, ctx_stride_row, ctx_stride_head,
                          ctx_stride_pos, heads, dim, dtype))
    return e;
  if (int e = check_cache("beam_attention (generated)", kg, vg, gen_rows, gen_len_cap, gen_stride_row,
                          gen_stride_head, gen_stride_pos, heads, dim, dtype))
    return e;
  const int64_t rows = (int64_t)groups * beams;
  if (groups > ctx_rows) return fail(OMNIASR_ERR_ARGUMENT, "%s: %d inputs, context cache has %lld rows", name, groups,
                                     (long long)ctx_rows);
  if (rows > gen_rows) return fail(OMNIASR_ERR_ARGUMENT, "%s: %lld rows, generated cache has %lld", name,
                                   (long long)rows, (long long)gen_rows);
  if (ctx_keys < 0 || ctx_keys > ctx_len_cap)
    return fail(OMNIASR_ERR_ARGUMENT, "%s: ctx_keys %d outside [0, %lld]", name, ctx_keys, (long long)ctx_len_cap);
  if (ptr_stride < gen_len_cap) return fail(OMNIASR_ERR_ARGUMENT, "%s: ptr row stride %lld < generated length %lld",
                                            name, (long long)ptr_stride, (long long)gen_len_cap);
  const omni::SplitPlan pg = omni::plan_split(dtype, dim, (int)rows, heads, 1, gen_len_cap);
  omni::SplitArgs b{};
  b.q = q;
  b.k = kg;
  b.v = vg;
  b.s_kb = gen_stride_row;
  b.s_kh = gen_stride_head;
  b.s_ks = gen_stride_pos;
  b.cache_rows = gen_rows;
  b.cache_len = gen_len_cap;
  b.lengths = gen_len;
  b.ptr = ptr;
  b.ptr_stride = ptr_stride;
  b.heads = heads;
  b.nq = 1;
  b.causal = 0;
  b.chunk = pg.chunk;
  b.qblocks = 1;
  b.key_bound = (int64_t)pg.splits * pg.chunk;
  b.qscale = scale * omni::kLog2e;
  b.status = status;
  if (omni::tc_path_enabled(dtype, dim, beams)) {
    // Context keys on the tensor cores (one read per input for all its beams); the generated keys, gathered
    // through the pointers, are attended by the combine itself while the pass runs, and merged with it.
    const int stc = omni::tc_segments(ctx_keys);
    const size_t need = omni::partial_bytes(rows, heads, stc, dim);
    if (!workspace || workspace_bytes < need || !aligned16(workspace))
      return fail(OMNIASR_ERR_WORKSPACE, "%s: workspace %zu bytes, %zu needed (16-byte aligned)", name,
                  workspace ? workspace_bytes : (size_t)0, need);
    omni::TcParams t{};
    t.q = static_cast<const __nv_bfloat16*>(q);
    t.lengths = ctx_len;
    t.groups = groups;
    t.nq = beams;
    t.causal = 0;
    t.heads = heads;
    t.dim = dim;
    t.qscale = scale * omni::kLog2e;
    t.status = status;
    omni::carve_partials(workspace, rows, heads, stc, dim, &t.part_o, &t.part_ml);
    if (int e = cuda_status(omni::launch_tc_pass(kc, vc, ctx_rows, ctx_len_cap, ctx_stride_row, ctx_stride_head,
                                                 ctx_stride_pos, ctx_keys, t, stream),
                            "context attention launch"))
      return e;
    omni::GenKeys gk{};
    gk.k = static_cast<const __nv_bfloat16*>(kg);
    gk.v = static_cast<const __nv_bfloat16*>(vg);
    gk.s_kb = gen_stride_row;
    gk.s_kh = gen_stride_head;
    gk.s_ks = gen_stride_pos;
    gk.cache_rows = gen_rows;
    gk.cache_len = gen_len_cap;
    gk.ptr = ptr;
    gk.ptr_stride = ptr_stride;
    gk.gen_len = gen_len;
    gk.enabled = 1;
    return cuda_status(omni::launch_tc_combine(t, out, gk, stream), "combine launch");
  }
  const omni::SplitPlan pc = omni::plan_split(dtype, dim, groups, heads, beams, ctx_keys);
  const int st = pc.splits + pg.splits;
  const size_t need = omni::partial_bytes(rows, heads, st, dim);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return fail(OMNIASR_ERR_WORKSPACE, "%s: workspace %zu bytes, %zu needed (16-byte aligned)", name,
                workspace ? workspace_bytes : (size_t)0, need);
  float *po, *pml;
  omni::carve_partials(workspace, rows, heads, st, dim, &po, &pml);
  omni::SplitArgs a{};
  a.q = q;
  a.k = kc;
  a.v = vc;
  a.s_kb = ctx_stride_row;
  a.s_kh = ctx_stride_head;
  a.s_ks = ctx_stride_pos;
  a.cache_rows = ctx_rows;
  a.cache_len = ctx_len_cap;
  a.lengths = ctx_len;
  a.part_o = po;
  a.part_ml = pml;
  a.st = st;
  a.sp_offset = 0;
  a.heads = heads;
  a.nq = beams;
  a.causal = 0;
  a.chunk = pc.chunk;
  a.qblocks = pc.qblocks;
  a.key_bound = (int64_t)pc.splits * pc.chunk;
  a.qscale = scale * omni::kLog2e;
  a.status = status;
  if (int e = cuda_status(omni::launch_split(dtype, dim, false, pc, a, groups, stream), "context split launch"))
    return e;
  b.part_o = po;
  b.part_ml = pml;
  b.st = st;
  b.sp_offset = pc.splits;
  if (int e = cuda_status(omni::launch_split(dtype, dim, true, pg, b, (int)rows, stream), "generated split launch"))
    return e;
  return cuda_status(omni::launch_combine(dtype, dim, po, pml, out, rows * heads, st, stream), "combine launch");
}

int omniasr_prefill_attention(const void* q, int64_t q_stride_row, int64_t q_stride_head, int64_t q_stride_pos,
                              const void* k, int64_t k_stride_row, int64_t k_stride_head, int64_t k_stride_pos,
                              const void* v, int64_t v_stride_row, int64_t v_stride_head, int64_t v_stride_pos,
                              void* out, int64_t out_stride_row, int64_t out_stride_head, int64_t out_stride_pos,
                              int batch, int heads, int width, int dim, float scale, int dtype, int* status,
                              cudaStream_t stream) {
  const char* name = "prefill_attention";
  if (dtype != OMNIASR_BF16 || (dim != 128 && dim != 512))
    return fail(OMNIASR_ERR_UNSUPPORTED, "%s: bf16 with head_dim 128 or 512 only (dtype %d, head_dim %d)", name, dtype,
                dim);
  if (int e = check_device()) return e;
  if (batch < 0 || heads <= 0 || width < 0) return fail(OMNIASR_ERR_ARGUMENT, "%s: shape", name);
  if (batch == 0 || width == 0) return ok();
  if (!q || !k || !v || !out) return fail(OMNIASR_ERR_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(out))
    return fail(OMNIASR_ERR_ARGUMENT, "%s: pointers must be 16-byte aligned", name);
  const int64_t strides[12] = {q_stride_row, q_stride_head, q_stride_pos, k_stride_row, k_stride_head, k_stride_pos,
                               v_stride_row, v_stride_head, v_stride_pos, out_stride_row, out_stride_head,
                               out_stride_pos};
  for (int64_t st : strides)
    if (!stride_ok(st, dtype)) return fail(OMNIASR_ERR_ARGUMENT, "%s: strides must keep 16-byte alignment", name);
  omni::PrefillArgs a;
  a.q = q;
  a.q_sb = q_stride_row;
  a.q_sh = q_stride_head;
  a.q_sw = q_stride_pos;
  a.k = k;
  a.k_sb = k_stride_row;
  a.k_sh = k_stride_head;
  a.k_sw = k_stride_pos;
  a.v = v;
  a.v_sb = v_stride_row;
  a.v_sh = v_stride_head;
  a.v_sw = v_stride_pos;
  a.out = out;
  a.o_sb = out_stride_row;
  a.o_sh = out_stride_head;
  a.o_sw = out_stride_pos;
  a.batch = batch;
  a.heads = heads;
  a.width = width;
  a.scale = scale;
  a.status = status;
  return cuda_status(dim == 512 ? omni::launch_prefill_wide(a, stream) : omni::launch_prefill(a, stream), "prefill launch");
}

size_t omniasr_prefill_grouped_workspace(int batch, int heads, int width, int dim) {
  if (batch <= 0 || heads <= 0 || width <= 0 || (dim != 128 && dim != 512)) return 0;
  return omni::tc_prefill_workspace(batch, heads, width, dim, kPrefillGroup);
}

int omniasr_prefill_attention_grouped(const void* q, const void* k_cache, const void* v_cache, int64_t cache_rows,
                                      int64_t cache_len, int64_t stride_row, int64_t stride_head, int64_t stride_pos,
                                      void* out, int batch, int heads, int width, int dim, float scale, int dtype,
                                      void* workspace, size_t workspace_bytes, int* status, cudaStream_t stream) {
  const char* name = "prefill_attention_grouped";
  if (dtype != OMNIASR_BF16 || (dim != 128 && dim != 512))
    return fail(OMNIASR_ERR_UNSUPPORTED, "%s: bf16 with head_dim 128 or 512 (dtype %d, head_dim %d)", name, dtype,
                dim);
  if (int e = check_common(dtype, dim, heads)) return e;
  if (batch < 0 || width < 0) return fail(OMNIASR_ERR_ARGUMENT, "%s: batch %d width %d", name, batch, width);
  if (batch == 0 || width == 0) return ok();
  if (!q || !out) return fail(OMNIASR_ERR_ARGUMENT, "%s: null pointer", name);
  if (!aligned16(q) || !aligned16(out)) return fail(OMNIASR_ERR_ARGUMENT, "%s: q / out not 16-byte aligned", name);
  if (int e = check_cache(name, k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head, stride_pos, heads,
                          dim, dtype))
    return e;
  if (batch > cache_rows || width > cache_len)
    return fail(OMNIASR_ERR_ARGUMENT, "%s: %d rows of width %d, cache [%lld rows, %lld positions]", name, batch,
                width, (long long)cache_rows, (long long)cache_len);
  const int gpr = (width + kPrefillGroup - 1) / kPrefillGroup;
  const int64_t groups = (int64_t)batch * gpr;
  if (groups * heads > omni::kCounterUnits)
    return fail(OMNIASR_ERR_ARGUMENT, "%s: %lld query groups x %d heads exceed %d units per call (split the batch)",
                name, (long long)groups, heads, omni::kCounterUnits);
  const size_t need = omniasr_prefill_grouped_workspace(batch, heads, width, dim);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return fail(OMNIASR_ERR_WORKSPACE, "%s: workspace %zu bytes, %zu needed (16-byte aligned)", name,
                workspace ? workspace_bytes : (size_t)0, need);
  omni::TcParams t{};
  t.q = static_cast<const __nv_bfloat16*>(q);
  t.lengths = nullptr;
  t.groups = (int)groups;
  t.nq = kPrefillGroup;
  t.causal = 1;
  t.heads = heads;
  t.dim = dim;
  t.kv_div = gpr;
  t.prefill = 1;
  t.st = omni::tc_prefill_segments(batch, heads, width, kPrefillGroup);
  t.qscale = scale * omni::kLog2e;
  t.status = status;
  t.out = static_cast<__nv_bfloat16*>(out);
  t.counters = static_cast<unsigned*>(workspace);
  omni::carve_partials(static_cast<char*>(workspace) + omni::kCounterBytes, (int64_t)omni::tc_grid() * 16, 1, t.st,
                       dim, &t.part_o, &t.part_ml);
  return cuda_status(omni::launch_tc_pass(k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head,
                                          stride_pos, width, t, stream),
                     "grouped prefill launch");
}

int omniasr_reorder_gather(const void* src, int64_t src_row_stride, int64_t src_rows, void* dst,
                           int64_t dst_row_stride, const void* parent, int parent_is_int64, int rows,
                           int64_t row_bytes, int* status, cudaStream_t stream) {
  if (int e = check_device()) return e;
  if (rows < 0 || row_bytes < 0 || src_rows < 0) return fail(OMNIASR_ERR_ARGUMENT, "reorder_gather: sizes");
  if (rows > 65535) return fail(OMNIASR_ERR_ARGUMENT, "reorder_gather: %d rows (at most 65535 per call)", rows);
  if (rows == 0 || row_bytes == 0) return ok();
  if (!src || !dst || !parent) return fail(OMNIASR_ERR_ARGUMENT, "reorder_gather: null pointer");
  if (src_row_stride < row_bytes && src_rows > 1) return fail(OMNIASR_ERR_ARGUMENT, "reorder_gather: src rows overlap");
  if (dst_row_stride < row_bytes && rows > 1) return fail(OMNIASR_ERR_ARGUMENT, "reorder_gather: dst rows overlap");
  const char* s0 = static_cast<const char*>(src);
  const char* s1 = s0 + (src_rows > 0 ? (src_rows - 1) * src_row_stride + row_bytes : 0);
  const char* d0 = static_cast<const char*>(dst);
  const char* d1 = d0 + (int64_t)(rows - 1) * dst_row_stride + row_bytes;
  if (d0 < s1 && s0 < d1) return fail(OMNIASR_ERR_ARGUMENT, "reorder_gather: src and dst overlap");
  omni::GatherArgs a;
  a.src = src;
  a.src_stride = src_row_stride;
  a.dst = dst;
  a.dst_stride = dst_row_stride;
  a.parent = parent;
  a.parent64 = parent_is_int64 ? 1 : 0;
  a.src_rows = src_rows;
  a.row_bytes = row_bytes;
  a.status = status;
  return cuda_status(omni::launch_gather(a, rows, stream), "reorder_gather launch");
}

int omniasr_propose(const int32_t* out, int64_t out_stride, int64_t out_cap, const int32_t* draft,
                    int64_t draft_stride, int64_t draft_cap, const int64_t* draft_len, const int64_t* last,
                    const int64_t* first, const int64_t* next, int64_t* start, int64_t* proposals,
                    uint8_t* use_draft, int rows, int tokens, int ngram, int behind, int ahead, const int* reach,
                    int self_window, int self_min, int* status, cudaStream_t stream) {
  if (int e = check_device()) return e;
  if (rows < 0 || rows > 65535) return fail(OMNIASR_ERR_ARGUMENT, "propose: rows %d", rows);
  if (rows == 0) return ok();
  if (!out || !draft || !draft_len || !last || !first || !next || !start || !proposals || !use_draft || !reach)
    return fail(OMNIASR_ERR_ARGUMENT, "propose: null pointer");
  if (tokens < 1 || ngram < 1 || ngram > omni::kProposeMaxNgram || behind < 0 || ahead < 0 || self_window < 1)
    return fail(OMNIASR_ERR_ARGUMENT, "propose: tokens %d, ngram %d (1..%d), behind %d, ahead %d, self_window %d",
                tokens, ngram, omni::kProposeMaxNgram, behind, ahead, self_window);
  int self_slots = 1;
  while (self_slots < self_window) self_slots <<= 1;  // as the reference's launch (kernels.py:372-373)
  if (behind + ahead + 1 > omni::kProposeMaxThreads || self_slots > omni::kProposeMaxThreads ||
      tokens > omni::kProposeMaxThreads)
    return fail(OMNIASR_ERR_UNSUPPORTED, "propose: at most %d draft candidates, own candidates and tokens",
                omni::kProposeMaxThreads);
  if (out_stride < 0 || draft_stride < 0 || out_cap < 1 || draft_cap < 0)
    return fail(OMNIASR_ERR_ARGUMENT, "propose: strides / capacities");
  omni::ProposeArgs a{};
  a.out = out;
  a.s_out = out_stride;
  a.out_cap = out_cap;
  a.draft = draft;
  a.s_draft = draft_stride;
  a.draft_cap = draft_cap;
  a.draft_len = draft_len;
  a.last = last;
  a.first = first;
  a.next = next;
  a.start = start;
  a.prop = proposals;
  a.use_draft = use_draft;
  a.tokens = tokens;
  a.ngram = ngram;
  a.behind = behind;
  a.ahead = ahead;
  a.self_slots = self_slots;
  a.self_min = self_min;
  for (int r = 0; r < 4; ++r) {
    a.reach_dist[r] = reach[2 * r];
    a.reach_need[r] = reach[2 * r + 1];
  }
  a.status = status;
  return cuda_status(omni::launch_propose(a, rows, stream), "propose launch");
}

int omniasr_accept(const int64_t* tokens, const int64_t* argmax, int32_t* out, int64_t out_stride, int64_t out_cap,
                   int64_t* tok, int64_t* last, uint8_t* done, int64_t* draft_next, const int64_t* start,
                   const uint8_t* use_draft, int rows, int width, int64_t limit, int64_t eos, int* status,
                   cudaStream_t stream) {
  if (int e = check_device()) return e;
  if (rows < 0 || width < 1 || width > 1024) return fail(OMNIASR_ERR_ARGUMENT, "accept: rows %d, width %d", rows, width);
  if (rows == 0) return ok();
  if (!tokens || !argmax || !out || !tok || !last || !done || !draft_next || !start || !use_draft)
    return fail(OMNIASR_ERR_ARGUMENT, "accept: null pointer");
  if (out_stride < 0 || out_cap < 1) return fail(OMNIASR_ERR_ARGUMENT, "accept: out stride / capacity");
  omni::AcceptArgs a{};
  a.tokens = tokens;
  a.argmax = argmax;
  a.out = out;
  a.s_out = out_stride;
  a.out_cap = out_cap;
  a.tok = tok;
  a.last = last;
  a.done = done;
  a.draft_next = draft_next;
  a.start = start;
  a.use_draft = use_draft;
  a.rows = rows;
  a.width = width;
  a.limit = limit;
  a.eos = eos;
  a.status = status;
  return cuda_status(omni::launch_accept(a, stream), "accept launch");
}

int omniasr_beam_select(const void* logp, int64_t logp_stride, int logp_is_f32, float* score, uint8_t* ended,
                        int64_t* count, int64_t* tok, int32_t* hist, int64_t hist_stride, int64_t hist_width,
                        int32_t* ptr, int64_t ptr_stride, int64_t ptr_width, int64_t* k_step, const int64_t* ctx,
                        uint8_t* gdone, int groups, int beams, int vocab, int length_norm, int64_t eos, int64_t pad,
                        int64_t limit, int* status, cudaStream_t stream) {
  if (int e = check_device()) return e;
  if (groups < 0 || beams < 1 || beams > omni::kBeamSelectMaxBeams || vocab < 1)
    return fail(OMNIASR_ERR_ARGUMENT, "beam_select: groups %d, beams %d (1..%d), vocab %d", groups, beams,
                omni::kBeamSelectMaxBeams, vocab);
  if ((int64_t)beams * vocab > INT32_MAX)
    return fail(OMNIASR_ERR_ARGUMENT, "beam_select: beams x vocab must fit in 31 bits");
  if (eos < 0 || eos >= vocab) return fail(OMNIASR_ERR_ARGUMENT, "beam_select: eos %lld outside the vocabulary",
                                           (long long)eos);
  if (logp_stride < vocab || hist_width < 1 || ptr_width < 0 || hist_stride < hist_width || ptr_stride < ptr_width)
    return fail(OMNIASR_ERR_ARGUMENT, "beam_select: strides / widths");
  if (groups == 0) return ok();
  if (!logp || !score || !ended || !count || !tok || !hist || (!ptr && ptr_width > 0) || !k_step || !ctx || !gdone)
    return fail(OMNIASR_ERR_ARGUMENT, "beam_select: null pointer");
  omni::BeamSelectArgs a{};
  a.logp = logp;
  a.s_logp = logp_stride;
  a.logp_f32 = logp_is_f32 ? 1 : 0;
  a.score = score;
  a.ended = ended;
  a.count = count;
  a.tok = tok;
  a.hist = hist;
  a.s_hist = hist_stride;
  a.hist_w = hist_width;
  a.ptr = ptr;
  a.s_ptr = ptr_stride;
  a.ptr_w = ptr_width;
  a.k_step = k_step;
  a.ctx = ctx;
  a.gdone = gdone;
  a.groups = groups;
  a.beams = beams;
  a.vocab = vocab;
  a.length_norm = length_norm ? 1 : 0;
  a.eos = eos;
  a.pad = pad;
  a.limit = limit;
  a.status = status;
  return cuda_status(omni::launch_beam_select(a, stream), "beam_select launch");
}

size_t omniasr_decode_gemm_workspace(int rows, int n, int k, int mode) {
  if (rows < 1 || rows > omni::kGemmMaxRows) return 0;
  return omni::gemm_workspace_bytes(rows, n, k, mode);
}

int omniasr_decode_gemm_rope(const void* x, int64_t x_stride, int rows, const void* w, int64_t w_stride, int k,
                             const float* cs, int64_t cs_positions, const int64_t* pos, const int64_t* slots,
                             const int64_t* cache_pos, void* q_out, void* k_cache, void* v_cache, int64_t cache_rows,
                             int64_t cache_len, int64_t stride_row, int64_t stride_head, int64_t stride_pos, int heads,
                             int dim, void* workspace, size_t workspace_bytes, int* status, cudaStream_t stream) {
  if (int e = check_device()) return e;
  if (rows < 0 || rows > omni::kGemmMaxRows || k < 0 || heads <= 0 || dim <= 0 || dim % 128 != 0)
    return fail(OMNIASR_ERR_ARGUMENT, "decode_gemm_rope: rows %d (at most %d), k %d, heads %d, dim %d (a multiple of "
                "128)", rows, omni::kGemmMaxRows, k, heads, dim);
  if (rows == 0) return ok();
  if (k == 0) return fail(OMNIASR_ERR_ARGUMENT, "decode_gemm_rope: k = 0");
  if (!x || !w || !workspace || !cs || !pos || !q_out) return fail(OMNIASR_ERR_ARGUMENT, "decode_gemm_rope: null pointer");
  if (!aligned16(x) || !aligned16(w) || !aligned16(workspace) || !aligned16(cs) || (x_stride * 2) % 16 ||
      (w_stride * 2) % 16 || x_stride < k || w_stride < k)
    return fail(OMNIASR_ERR_ARGUMENT, "decode_gemm_rope: x / w / cs must be 16-byte aligned, row strides >= k");
  if (int e = check_cache("decode_gemm_rope", k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head,
                          stride_pos, heads, dim, OMNIASR_BF16))
    return e;
  const int n = 3 * heads * dim;
  if (omni::gemm_tiles(n, omni::kGemmStore) > omni::kGemmMaxTiles)
    return fail(OMNIASR_ERR_UNSUPPORTED, "decode_gemm_rope: n %d needs more than %d weight tiles", n,
                omni::kGemmMaxTiles);
  const size_t need = omni::gemm_workspace_bytes(rows, n, k, omni::kGemmStore);
  if (workspace_bytes < need)
    return fail(OMNIASR_ERR_WORKSPACE, "decode_gemm_rope: workspace %zu bytes, %zu needed", workspace_bytes, need);
  omni::GemmArgs a{};
  a.rows = rows;
  a.n = n;
  a.k = k;
  a.mode = omni::kGemmRope;
  a.status = status;
  a.head_dim = dim;
  a.rope.cs = cs;
  a.rope.cs_positions = cs_positions;
  a.rope.pos = pos;
  a.rope.slots = slots;
  a.rope.cache_pos = cache_pos;
  a.rope.q_out = q_out;
  a.rope.k_cache = k_cache;
  a.rope.v_cache = v_cache;
  a.rope.s_kb = stride_row;
  a.rope.s_kh = stride_head;
  a.rope.s_ks = stride_pos;
  a.rope.cache_rows = cache_rows;
  a.rope.cache_len = cache_len;
  a.rope.heads = heads;
  a.rope.status = status;
  return cuda_status(omni::launch_decode_gemm(x, x_stride, w, w_stride, a, workspace, workspace_bytes, stream),
                     "decode_gemm_rope launch");
}

int omniasr_decode_gemm(const void* x, int64_t x_stride, int rows, const void* w, int64_t w_stride, int n, int k,
                        int mode, const void* residual, int64_t residual_stride, void* y, int64_t y_stride,
                        void* workspace, size_t workspace_bytes, int* status, cudaStream_t stream) {
  if (int e = check_device()) return e;
  if (rows < 0 || rows > omni::kGemmMaxRows || n < 0 || k < 0)
    return fail(OMNIASR_ERR_ARGUMENT, "decode_gemm: rows %d (at most %d), n %d, k %d", rows, omni::kGemmMaxRows, n, k);
  if (rows == 0 || n == 0) return ok();
  if (k == 0) return fail(OMNIASR_ERR_ARGUMENT, "decode_gemm: k = 0");
  if (mode != omni::kGemmStore && mode != omni::kGemmResidual && mode != omni::kGemmSwiglu)
    return fail(OMNIASR_ERR_ARGUMENT, "decode_gemm: mode %d", mode);
  if (!x || !w || !y || !workspace) return fail(OMNIASR_ERR_ARGUMENT, "decode_gemm: null pointer");
  if (mode == omni::kGemmResidual && !residual) return fail(OMNIASR_ERR_ARGUMENT, "decode_gemm: no residual");
  if (!aligned16(x) || !aligned16(w) || !aligned16(workspace) || (x_stride * 2) % 16 || (w_stride * 2) % 16 ||
      x_stride < k || w_stride < k)
    return fail(OMNIASR_ERR_ARGUMENT, "decode_gemm: x / w must be 16-byte aligned with row strides >= k keeping it");
  if (y_stride < n || (mode == omni::kGemmResidual && residual_stride < n))
    return fail(OMNIASR_ERR_ARGUMENT, "decode_gemm: output / residual row stride < n");
  if (omni::gemm_tiles(n, mode) > omni::kGemmMaxTiles)
    return fail(OMNIASR_ERR_UNSUPPORTED, "decode_gemm: n %d needs more than %d weight tiles", n, omni::kGemmMaxTiles);
  const size_t need = omni::gemm_workspace_bytes(rows, n, k, mode);
  if (workspace_bytes < need)
    return fail(OMNIASR_ERR_WORKSPACE, "decode_gemm: workspace %zu bytes, %zu needed", workspace_bytes, need);
  omni::GemmArgs a{};
  a.rows = rows;
  a.n = n;
  a.k = k;
  a.mode = mode;
  a.residual = static_cast<const __nv_bfloat16*>(residual);
  a.ld_res = residual_stride;
  a.y = static_cast<__nv_bfloat16*>(y);
  a.ld_y = y_stride;
  a.status = status;
  return cuda_status(omni::launch_decode_gemm(x, x_stride, w, w_stride, a, workspace, workspace_bytes, stream),
                     "decode_gemm launch");
}

}  // extern "C"
