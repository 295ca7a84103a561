/* omniASR-LLM decoder attention hot path on B200 (sm_100a): the C ABI.
 *
 * Every entry point takes plain device pointers, element strides, host ints and a CUDA stream,
 * launches asynchronously on that stream, never synchronises, never allocates, and returns
 * OMNIASR_OK or an error code (omniasr_last_error() has the message). Launch grids depend only on
 * host ints, so every call can be captured in a CUDA graph; lengths, positions and pointers are
 * read on the device.
 *
 * Tensors: `dtype` is OMNIASR_BF16 or OMNIASR_F32 for q / k / v / out; head_dim (`dim`) is one of
 * 16, 32, 64, 128, 256, 512; the innermost (head_dim) stride of every tensor is 1, the other
 * strides are in elements and every pointer / stride must keep 16-byte alignment. Caches are
 * [rows, heads, len, dim] with strides (stride_row, stride_head, stride_pos); k and v caches of
 * one call share their strides. Index tensors (lengths, positions, slots) are int64.
 *
 * `status` (may be NULL) is a device int the kernels OR error bits into: 1 = an index read from a
 * tensor (length, position, slot, beam pointer, parent) was outside its tensor and the access was
 * skipped; 2 = a bounded device wait gave up; 4 = a kernel found its shared memory not laid out as it
 * requires and did nothing. The kernels never trap.
 *
 * Each declaration names the function of the reference (Wataru-Nakata/omniasr-trt, Python) it
 * replaces, as path:line within that project.
 */
#ifndef OMNIASR_B200_H
#define OMNIASR_B200_H

#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define OMNIASR_BF16 0
#define OMNIASR_F32 1

#define OMNIASR_OK 0
#define OMNIASR_ERR_ARGUMENT 1    /* a shape, stride, pointer alignment or size is invalid */
#define OMNIASR_ERR_UNSUPPORTED 2 /* dtype or head_dim not supported */
#define OMNIASR_ERR_WORKSPACE 3   /* workspace smaller than omniasr_attention_workspace() */
#define OMNIASR_ERR_CUDA 4        /* a CUDA launch failed */
#define OMNIASR_ERR_DEVICE 5      /* the current device cannot run sm_100a code */

/* Workspace kinds for omniasr_attention_workspace(). */
#define OMNIASR_DECODE 0
#define OMNIASR_DRAFT 1
#define OMNIASR_BEAM 2

/* Version of this ABI (bumped on any signature change). */
int omniasr_abi_version(void);

/* Message of the last error returned on this host thread ("" if none). */
const char* omniasr_last_error(void);

/* 1 if `device` can run this library's kernels (compute capability 10.0), else 0.
 * Replaces omniasr_trt/kernels.py:25-26 (`available`). */
int omniasr_device_supported(int device);

/* The reference's split rule: key splits (a power of two, about `programs` programs in all) and
 * the keys each split covers. Host only. Replaces omniasr_trt/kernels.py:393-400 (`splits_for`). */
int omniasr_splits_for(int rows, int heads, int keys, int block, int programs, int* splits, int* chunk);

/* Bytes of workspace an attention call of this shape needs on the current device (the split
 * partials; the reference allocates them inside its wrappers, omniasr_trt/kernels.py:319-320,
 * :349-350, :416-417). kind: OMNIASR_DECODE (per_group = 1), OMNIASR_DRAFT (per_group = tokens),
 * OMNIASR_BEAM (per_group = beams, gen_keys = generated-cache length).
 *
 * Decode and draft workspaces begin with OMNIASR_ATTENTION_COUNTER_BYTES of per-(row, head) counters
 * through which the last CTA to finish a row's keys merges the partial results itself (no second
 * kernel). Those bytes must be zero before the workspace's first use, and every call leaves them
 * zero: zero a workspace once when allocating it and reuse it for calls in stream order. Calls that
 * may overlap on the GPU need workspaces of their own. After status bit 2 (a wait gave up) the
 * counters may be left non-zero: zero them again. The beam workspace has no counters. */
#define OMNIASR_ATTENTION_COUNTER_BYTES 65536
size_t omniasr_attention_workspace(int kind, int dtype, int groups, int per_group, int heads, int dim,
                                   int64_t keys, int64_t gen_keys);

/* RoPE of q and k at pos[n] (interleaved pairs, fp32, table cs [cs_positions, dim/2, 2] fp32) and
 * the KV-cache append: rotated k and raw v of token n written at cache row slots[n] (NULL: n) and
 * position cache_pos[n] (NULL: pos[n]); rotated q written to q_out [n, heads, dim] contiguous.
 * qkv is [n, 3 * heads * dim] with row stride qkv_stride. Bit-exact with the reference.
 * Replaces omniasr_trt/kernels.py:294-306 (`rope_kv`) and its kernel kernels.py:31-54. */
int omniasr_rope_kv(const void* qkv, int64_t qkv_stride, const float* cs, int64_t cs_positions, const int64_t* pos,
                    const int64_t* slots, const int64_t* cache_pos, void* q_out, void* k_cache, void* v_cache,
                    int64_t cache_rows, int64_t cache_len, int64_t stride_row, int64_t stride_head,
                    int64_t stride_pos, int n, int heads, int dim, int dtype, int* status, cudaStream_t stream);

/* Flash-decode: q [batch, heads, dim] contiguous, row b attends to keys [0, lengths[b]) of cache
 * row b (all within the first `keys`, which fixes the grid); out [batch, heads, dim] contiguous in
 * q's dtype. A row of length 0 gets zeros.
 * Replaces omniasr_trt/kernels.py:406-423 (`decode_attention`: _attn_split + _attn_combine). */
int omniasr_decode_attention(const void* q, const void* k_cache, const void* v_cache, int64_t cache_rows,
                             int64_t cache_len, int64_t stride_row, int64_t stride_head, int64_t stride_pos,
                             const int64_t* lengths, void* out, int batch, int heads, int dim, int keys, float scale,
                             int dtype, void* workspace, size_t workspace_bytes, int* status, cudaStream_t stream);

/* Draft verification: q [batch * tokens, heads, dim], row b's queries at rows b*tokens ..
 * b*tokens + tokens - 1; query i of row b attends to keys [0, lengths[b] + i) of cache row b (all
 * within the first `keys`). out like q.
 * Replaces omniasr_trt/kernels.py:338-358 (`draft_attention`: _beam_ctx CAUSAL + _beam_combine). */
int omniasr_draft_attention(const void* q, const void* k_cache, const void* v_cache, int64_t cache_rows,
                            int64_t cache_len, int64_t stride_row, int64_t stride_head, int64_t stride_pos,
                            const int64_t* lengths, void* out, int batch, int tokens, int heads, int dim, int keys,
                            float scale, int dtype, void* workspace, size_t workspace_bytes, int* status,
                            cudaStream_t stream);

/* Beam attention: q [groups * beams, heads, dim] (input g's beams at rows g*beams ..); row r
 * attends to its input's context keys [0, ctx_len[g]) of kc/vc row g (all within `ctx_keys`) and
 * to its generated keys j < gen_len[r], key j read from kg/vg row ptr[r * ptr_stride + j] (int32)
 * at position j. out like q; a row with no keys gets zeros.
 * Replaces omniasr_trt/kernels.py:309-332 (`beam_attention`: _beam_ctx + _beam_gen + _beam_combine). */
int omniasr_beam_attention(const void* q, const void* kc, const void* vc, int64_t ctx_rows, int64_t ctx_len_cap,
                           int64_t ctx_stride_row, int64_t ctx_stride_head, int64_t ctx_stride_pos,
                           const int64_t* ctx_len, const void* kg, const void* vg, int64_t gen_rows,
                           int64_t gen_len_cap, int64_t gen_stride_row, int64_t gen_stride_head,
                           int64_t gen_stride_pos, const int32_t* ptr, int64_t ptr_stride, const int64_t* gen_len,
                           void* out, int groups, int beams, int heads, int dim, int ctx_keys, float scale, int dtype,
                           void* workspace, size_t workspace_bytes, int* status, cudaStream_t stream);

/* Causal prefill attention (bf16, head_dim 128 or 512): out[b, h, w] = softmax(q[b, h, w] . k[b, h, :w+1]^T *
 * scale) . v[b, h, :w+1] for every position w < width. q, k, v and out are [batch, heads, width, dim] given by base
 * pointer and (row, head, position) element strides (k and v are typically views of the KV cache; out may be a
 * [batch, width, heads, dim] buffer seen through its strides). Replaces the reference's prefill
 * F.scaled_dot_product_attention(q, k, v, is_causal=True), omniasr_trt/decode.py:171. */
int omniasr_prefill_attention(const void* q, int64_t q_stride_row, int64_t q_stride_head, int64_t q_stride_pos,
                              const void* k, int64_t k_stride_row, int64_t k_stride_head, int64_t k_stride_pos,
                              const void* v, int64_t v_stride_row, int64_t v_stride_head, int64_t v_stride_pos,
                              void* out, int64_t out_stride_row, int64_t out_stride_head, int64_t out_stride_pos,
                              int batch, int heads, int width, int dim, float scale, int dtype, int* status,
                              cudaStream_t stream);

/* Causal prefill attention on the tensor-core decode pass, for head_dims without a dedicated prefill kernel (the
 * shipped model's 512; 128 also works): each batch row's `width` query positions are cut into groups of 16
 * consecutive positions, group j attending, as a 16-token draft, to keys [0, 16j + 1 + i) of the row's cache.
 * q and out are [batch * wp, heads, dim] contiguous with wp = width rounded up to a multiple of 16 (row b's query w
 * at row b * wp + w; the padding rows are computed and may be ignored); k_cache / v_cache are [>= batch, heads,
 * >= width, dim] views as for omniasr_draft_attention. batch * (wp / 16) * heads <= 16384 per call. The workspace
 * (omniasr_prefill_grouped_workspace() bytes) starts with unit counters that must be zero on entry; every call leaves
 * them zero. Replaces, like omniasr_prefill_attention, the prefill's F.scaled_dot_product_attention(q, k, v,
 * is_causal=True) of omniasr_trt/decode.py:171. */
size_t omniasr_prefill_grouped_workspace(int batch, int heads, int width, int dim);
int omniasr_prefill_attention_grouped(const void* q, const void* k_cache, const void* v_cache, int64_t cache_rows,
                                      int64_t cache_len, int64_t stride_row, int64_t stride_head, int64_t stride_pos,
                                      void* out, int batch, int heads, int width, int dim, float scale, int dtype,
                                      void* workspace, size_t workspace_bytes, int* status, cudaStream_t stream);

/* Beam reorder: dst row r (r < rows <= 65535) = src row parent[r], byte-exact; rows are row_bytes long,
 * strides in bytes; parent is int32 (parent_is_int64 = 0) or int64. src and dst must not overlap.
 * Replaces the K/V `index_select(0, parent)` of omniasr_trt/llm.py:237-238 and the pointer /
 * history gathers `ptr[parent]`, `hist[parent]` of omniasr_trt/beam.py:175-176. */
int omniasr_reorder_gather(const void* src, int64_t src_row_stride, int64_t src_rows, void* dst,
                           int64_t dst_row_stride, const void* parent, int parent_is_int64, int rows,
                           int64_t row_bytes, int* status, cudaStream_t stream);

/* Speculative decoding's proposal for rows 0..rows-1: `tokens` proposed tokens per row (int64 `proposals`
 * [rows, tokens]), whether they come from the draft (`use_draft`, one byte per row) and the draft position of the
 * first (`start`). `out` holds each row's tokens by position (int32, row stride `out_stride` elements, `out_cap`
 * positions), `draft` its draft (int32, `draft_stride`, `draft_cap`); `draft_len`, `last` (position of the newest
 * token), `first` (position of the segment's first) and `next` (draft position expected after the newest) are
 * int64 per row. `reach` holds 4 (distance, matching tokens needed) pairs. Bit-exact with
 * omniasr_trt/kernels.py:361-377 (`propose`: _propose, :214-262). */
int omniasr_propose(const int32_t* out, int64_t out_stride, int64_t out_cap, const int32_t* draft,
                    int64_t draft_stride, int64_t draft_cap, const int64_t* draft_len, const int64_t* last,
                    const int64_t* first, const int64_t* next, int64_t* start, int64_t* proposals,
                    uint8_t* use_draft, int rows, int tokens, int ngram, int behind, int ahead, const int* reach,
                    int self_window, int self_min, int* status, cudaStream_t stream);

/* Beam search's selection step after the LM head, in place on the first `groups` groups of `beams` rows
 * (beams <= 16; row r belongs to group r / beams). `logp` [groups * beams, vocab] holds the rows' log-probabilities
 * (bf16: logp_is_f32 = 0, or fp32; row stride `logp_stride` elements). Per group the best `beams` of its
 * beams x vocab candidates -- score + logp, or with `length_norm` (when the group's row 0 has counted tokens)
 * (score * count + logp) / (count + 1), each step rounded to fp32; an ended row offers only `eos` at its score --
 * in torch.topk(sorted=True)'s order (value descending, equal values by index ascending); then every row of a group
 * that is not done follows its parent: its `ptr` [rows, ptr_width] and `hist` [rows, hist_width] rows (int32, row
 * strides in elements) become the parent's, hist[row, k_step[group]] its new token, and score (fp32), count,
 * ended (one byte), tok (int64) the parent's updated ones; k_step and gdone (int64 / one byte per group, with
 * `ctx` the group's context length and `limit` the position cap) advance. Bit-exact with the tail of
 * omniasr_trt/beam.py:161-187 (BeamDecoder.step_beam after the log-softmax). */
int omniasr_beam_select(const void* logp, int64_t logp_stride, int logp_is_f32, float* score, uint8_t* ended,
                        int64_t* count, int64_t* tok, int32_t* hist, int64_t hist_stride, int64_t hist_width,
                        int32_t* ptr, int64_t ptr_stride, int64_t ptr_width, int64_t* k_step, const int64_t* ctx,
                        uint8_t* gdone, int groups, int beams, int vocab, int length_norm, int64_t eos, int64_t pad,
                        int64_t limit, int* status, cudaStream_t stream);

/* After a drafted step, in place on rows 0..rows-1: `tokens` [rows, width] were fed (the newest token, then the
 * proposal) and `argmax` [rows, width] is the greedy token after each (int64). A running row (done == 0) keeps
 * argmax 0..n at positions last+1+j of `out` (n: its leading proposed tokens equal to the argmax before them, cut
 * at the first EOS or position >= limit among those), and advances tok, last, done and draft_next (from `start`
 * when use_draft). Bit-exact with omniasr_trt/kernels.py:380-391 (`accept`: _accept, :264-291). */
int omniasr_accept(const int64_t* tokens, const int64_t* argmax, int32_t* out, int64_t out_stride, int64_t out_cap,
                   int64_t* tok, int64_t* last, uint8_t* done, int64_t* draft_next, const int64_t* start,
                   const uint8_t* use_draft, int rows, int width, int64_t limit, int64_t eos, int* status,
                   cudaStream_t stream);

/* Decode-time weight GEMM for the step's few token rows (rows <= 64), bf16 in and out, fp32 accumulate:
 *   OMNIASR_GEMM_STORE     y[m, j] = x[m, :] . w[j, :]                           (n rows of w)
 *   OMNIASR_GEMM_RESIDUAL  y[m, j] = residual[m, j] + x[m, :] . w[j, :]          (torch.addmm(residual, x, w.t()))
 *   OMNIASR_GEMM_SWIGLU    w = [gate; inner] (2n rows): y[m, j] = inner * silu(gate), each rounded to bf16 first
 * x [rows, k] and w row-major with element row strides (16-byte aligned rows); y / residual [rows, n]. The
 * workspace (omniasr_decode_gemm_workspace() bytes, 16-byte aligned) starts with per-tile arrival counters that
 * must be ZERO when a call starts (the partial tiles after them need no initial value); every call that completes
 * leaves them zero again, so a caller zeroes a workspace once and keeps it (one per stream: calls sharing a
 * workspace must not overlap on the GPU; after status bit 2 they may be left non-zero: zero or replace it). The kernel
 * is launched as a programmatic dependent and requests its first weight tiles before waiting for the kernel before
 * it, so w must not be written by the kernel launched just before on the same stream (x and the residual may be). Replaces the decoder step's weight GEMMs
 * of omniasr_trt/decode.py:201-205 / spec.py:100-107 (`qkv = norm(h) @ qkv_w.t()`, `torch.addmm(h, o, out_w.t())`,
 * `(norm(h) @ gi_w.t()).chunk(2)` + `inner * F.silu(gate)`, `torch.addmm(h, ..., ffo_w.t())`), which the reference
 * leaves to cuBLAS. */
#define OMNIASR_GEMM_STORE 0
#define OMNIASR_GEMM_RESIDUAL 1
#define OMNIASR_GEMM_SWIGLU 2
size_t omniasr_decode_gemm_workspace(int rows, int n, int k, int mode);
int omniasr_decode_gemm(const void* x, int64_t x_stride, int rows, const void* w, int64_t w_stride, int n, int k,
                        int mode, const void* residual, int64_t residual_stride, void* y, int64_t y_stride,
                        void* workspace, size_t workspace_bytes, int* status, cudaStream_t stream);

/* The QKV product of the decoder step with RoPE and the KV-cache append in its epilogue (bf16, rows <= 64): the
 * product qkv = x . w^T (w [3 * heads * dim, k]) is formed, each value rounded to bf16 as the GEMM's output would
 * be, and then handled as omniasr_rope_kv() handles a qkv row -- q rotated into q_out [rows, heads, dim], k rotated
 * and v as it is written into the caches at cache row slots[m] (or m) and position cache_pos[m] (or pos[m]) -- without
 * qkv ever reaching memory. Arguments as omniasr_decode_gemm() and omniasr_rope_kv(); the workspace is sized by
 * omniasr_decode_gemm_workspace(rows, 3 * heads * dim, k, OMNIASR_GEMM_STORE) and follows the same counter rule;
 * w likewise must not be written by the kernel launched just before on the same stream.
 * dim must be a multiple of 128. Replaces `qkv = norm(h) @ qkv_w.t()` followed by kernels.rope_kv
 * (omniasr_trt/decode.py:201-203, spec.py:100-101). */
int omniasr_decode_gemm_rope(const void* x, int64_t x_stride, int rows, const void* w, int64_t w_stride, int k,
                             const float* cs, int64_t cs_positions, const int64_t* pos, const int64_t* slots,
                             const int64_t* cache_pos, void* q_out, void* k_cache, void* v_cache, int64_t cache_rows,
                             int64_t cache_len, int64_t stride_row, int64_t stride_head, int64_t stride_pos, int heads,
                             int dim, void* workspace, size_t workspace_bytes, int* status, cudaStream_t stream);

/* Flash-decode for callers that cannot allocate device memory (no counterpart in the reference, whose
 * wrappers allocate their partials with torch.empty): the same computation and arguments as
 * omniasr_decode_attention() minus the workspace, which here is a device array inside this library of
 * omniasr_noalloc_scratch_bytes() bytes (8 MiB), held on every GPU that loads the library until the process
 * exits. For a host whose device memory is owned by another allocator, or a plugin interface that hands over
 * only the input and output buffers. Arguments are checked as by omniasr_decode_attention(); shapes whose split
 * partials exceed the array are then rejected with OMNIASR_ERR_WORKSPACE. The first call on a device (and again
 * after the device's context is recreated, e.g. by cudaDeviceReset) looks up the array's address with
 * cudaGetSymbolAddress and should come before any stream capture. All calls on a device share the array: calls
 * whose kernels overlap on the GPU race, so order them (same stream, or events). The array's leading unit
 * counters start at zero (a static device array is zero-initialised when the library loads) and every call that
 * completes normally leaves them zero; after a call that raised status bit 2 (a bounded wait gave up) they may
 * not be, so call omniasr_noalloc_reset() on the stream before the next no-alloc call. */
int omniasr_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache, int64_t cache_rows,
                                     int64_t cache_len, int64_t stride_row, int64_t stride_head, int64_t stride_pos,
                                     const int64_t* lengths, void* out, int batch, int heads, int dim, int keys,
                                     float scale, int dtype, int* status, cudaStream_t stream);

/* Size in bytes of the device scratch array behind omniasr_decode_attention_noalloc(). */
size_t omniasr_noalloc_scratch_bytes(void);

/* Zeroes the unit counters at the head of the current device's no-alloc scratch array, in stream order
 * (cudaMemsetAsync on the array itself; nothing is allocated). Needed only after a no-alloc call raised status
 * bit 2. No counterpart in the reference. */
int omniasr_noalloc_reset(cudaStream_t stream);

/* Self-test of the bounded device wait every kernel here uses (no counterpart in the reference): one kernel waits
 * on an mbarrier that nothing completes, gives up after limit_ns (0 < limit_ns <= 1e8), ORs the timeout bit (2)
 * into *status and returns; *waited_ns (may be NULL; device memory) gets the time it waited. The context stays
 * usable. */
int omniasr_selftest_wait_timeout(int64_t limit_ns, int* status, unsigned long long* waited_ns, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* OMNIASR_B200_H */
