// Flash-decode attention for callers that cannot allocate device memory.
//
// omniasr_decode_attention() needs a workspace for its split partials, and the caller allocates it. Some
// callers cannot: a host whose device memory is owned by another allocator (a serving engine that reserves
// the whole HBM for its own pool and hands kernels only tensors it already holds), or a plugin boundary
// whose interface passes just the input and output buffers (a C / cgo / ctypes caller with no way to ask the
// framework for scratch). omniasr_decode_attention_noalloc() serves them: the partials live in a file-scope
// device array, kNoAllocScratchBytes long, that the library's module carries on every GPU that loads it
// (held until the process exits); the call itself allocates nothing.
//
// Set-up: the first call on a device, with that device current, looks up the array's device address with
// cudaGetSymbolAddress (a host-side symbol is not a device pointer) and caches it for that device and its
// current context; make that first call outside any stream capture. A later call on the same device and context
// reuses the cached address; a new context on the device (after cudaDeviceReset) gets a fresh lookup.
//
// Sharing: all calls on a device use the same array and it keeps the previous call's contents. Only its
// leading unit counters must start at zero: a static device array is zero-initialised when the module loads,
// and every call that completes normally leaves the counters zero (a call writes every partial it reads before
// reading it). A call whose bounded wait gave up (status bit 2) may leave counters non-zero: the caller then
// runs omniasr_noalloc_reset() on the stream before the next call. Two calls whose kernels overlap on the GPU
// (different streams without ordering) race on the array: order them.

#include <stdio.h>

#include <mutex>

#include "attention.cuh"
#include "omniasr_b200.h"

namespace omni {
int set_last_error(int code, const char* message);  // capi.cu
int check_group_args(const char* name, const void* q, const void* k_cache, const void* v_cache, int64_t cache_rows,
                     int64_t cache_len, int64_t stride_row, int64_t stride_head, int64_t stride_pos,
                     const int64_t* lengths, const void* out, int groups, int nq, int heads, int dim, int keys,
                     int dtype);  // capi.cu
}

namespace {

// 8 MiB: the split partials of e.g. 8 rows x 32 heads over up to 4096 keys (bf16, head_dim 128).
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
struct Slot {
  void* ptr;
  void* ctx;  // the driver context the address belongs to
};
Slot g_scratch[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// The calling thread's current driver context (CUcontext), through the runtime's driver entry point (this library
// links only the runtime); null if it cannot be read.
void* current_context() {
  using GetCtx = int (*)(void**);
  static GetCtx fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return (GetCtx) nullptr;
    return reinterpret_cast<GetCtx>(f);
  }();
  void* ctx = nullptr;
  if (!fn || fn(&ctx) != 0) return nullptr;
  return ctx;
}

// Device address of the current device's scratch array (looked up once per device and context), or null.
void* scratch_address(cudaError_t* err, int* code, const char** what) {
  int device = 0;
  *err = cudaGetDevice(&device);
  if (*err != cudaSuccess || device < 0 || device >= kMaxDevices) {
    *code = OMNIASR_ERR_DEVICE;
    *what = "no usable current device";
    return nullptr;
  }
  void* ctx = current_context();
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  Slot& s = g_scratch[device];
  if (!s.ptr || s.ctx != ctx || !ctx) {
    void* ptr = nullptr;
    *err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (*err != cudaSuccess) {
      *code = OMNIASR_ERR_CUDA;
      *what = "scratch address lookup (cudaGetSymbolAddress) failed";
      return nullptr;
    }
    s.ptr = ptr;
    s.ctx = ctx;
  }
  *err = cudaSuccess;
  return s.ptr;
}

int lookup_failed(const char* fn, int code, const char* what, cudaError_t err) {
  char msg[256];
  snprintf(msg, sizeof msg, "%s: %s (%s)", fn, what, cudaGetErrorString(err));
  return omni::set_last_error(code, msg);
}

}  // namespace

extern "C" size_t omniasr_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int omniasr_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                                int64_t cache_rows, int64_t cache_len, int64_t stride_row,
                                                int64_t stride_head, int64_t stride_pos, const int64_t* lengths,
                                                void* out, int batch, int heads, int dim, int keys, float scale,
                                                int dtype, int* status, cudaStream_t stream) {
  // The regular entry point's argument checks come first, so a bad call reports the argument, not the scratch.
  if (int e = omni::check_group_args("decode_attention_noalloc", q, k_cache, v_cache, cache_rows, cache_len,
                                     stride_row, stride_head, stride_pos, lengths, out, batch, 1, heads, dim, keys,
                                     dtype))
    return e;
  if (batch == 0) return omni::set_last_error(OMNIASR_OK, "");
  const size_t need = omniasr_attention_workspace(OMNIASR_DECODE, dtype, batch, 1, heads, dim, (int64_t)keys, 0);
  if (need > kNoAllocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof msg,
             "decode_attention_noalloc: %d rows x %d heads x %d keys need %zu bytes of scratch; the no-alloc entry "
             "point holds %zu (use omniasr_decode_attention with a workspace)",
             batch, heads, keys, need, kNoAllocScratchBytes);
    return omni::set_last_error(OMNIASR_ERR_WORKSPACE, msg);
  }
  cudaError_t err = cudaSuccess;
  int code = OMNIASR_OK;
  const char* what = "";
  void* scratch = scratch_address(&err, &code, &what);
  if (!scratch) return lookup_failed("decode_attention_noalloc", code, what, err);
  return omniasr_decode_attention(q, k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head, stride_pos,
                                  lengths, out, batch, heads, dim, keys, scale, dtype, scratch, kNoAllocScratchBytes,
                                  status, stream);
}

extern "C" int omniasr_noalloc_reset(cudaStream_t stream) {
  static_assert(omni::kCounterBytes <= kNoAllocScratchBytes, "the counters lie inside the scratch array");
  cudaError_t err = cudaSuccess;
  int code = OMNIASR_OK;
  const char* what = "";
  void* scratch = scratch_address(&err, &code, &what);
  if (!scratch) return lookup_failed("noalloc_reset", code, what, err);
  err = cudaMemsetAsync(scratch, 0, omni::kCounterBytes, stream);  // writes the array in place; allocates nothing
  if (err != cudaSuccess) return lookup_failed("noalloc_reset", OMNIASR_ERR_CUDA, "cudaMemsetAsync failed", err);
  return omni::set_last_error(OMNIASR_OK, "");
}
