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
// cudaGetSymbolAddress (a host-side symbol is not a device pointer) and caches it per device; make that first
// call outside any stream capture. Every later call on the device reuses the cached address.
//
// Sharing: all calls on a device use the same array and it keeps the previous call's contents. Only its
// leading unit counters must start at zero: a static device array is zero-initialised when the module loads,
// and every call leaves the counters zero (a call writes every partial it reads before reading it). Two calls
// whose kernels overlap on the GPU (different streams without ordering) race on the array: order them.

#include <stdio.h>

#include <mutex>

#include "omniasr_b200.h"

namespace omni {
int set_last_error(int code, const char* message);  // capi.cu
}

namespace {

// 8 MiB: the split partials of e.g. 8 rows x 32 heads over up to 4096 keys (bf16, head_dim 128).
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
void* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// Device address of this device's scratch array (looked up once per device), or null.
void* scratch_address(int device, cudaError_t* err) {
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[device]) {
    void* ptr = nullptr;
    *err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (*err != cudaSuccess) return nullptr;
    g_scratch_ptr[device] = ptr;
  }
  *err = cudaSuccess;
  return g_scratch_ptr[device];
}

}  // namespace

extern "C" size_t omniasr_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int omniasr_decode_attention_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                                int64_t cache_rows, int64_t cache_len, int64_t stride_row,
                                                int64_t stride_head, int64_t stride_pos, const int64_t* lengths,
                                                void* out, int batch, int heads, int dim, int keys, float scale,
                                                int dtype, int* status, cudaStream_t stream) {
  if (batch <= 0) {
    // Nothing to launch; the regular entry point handles (and checks) this case without a workspace.
    return omniasr_decode_attention(q, k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head, stride_pos,
                                    lengths, out, batch, heads, dim, keys, scale, dtype, nullptr, 0, status, stream);
  }
  const size_t need =
      omniasr_attention_workspace(OMNIASR_DECODE, dtype, batch, 1, heads, dim, (int64_t)keys, 0);
  if (need == 0 || need > kNoAllocScratchBytes) {
    if (need == 0)  // an unsupported shape: the regular entry point reports it
      return omniasr_decode_attention(q, k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head,
                                      stride_pos, lengths, out, batch, heads, dim, keys, scale, dtype, nullptr, 0,
                                      status, stream);
    char msg[256];
    snprintf(msg, sizeof msg,
             "decode_attention_noalloc: %d rows x %d heads x %d keys need %zu bytes of scratch; the no-alloc entry "
             "point holds %zu (use omniasr_decode_attention with a workspace)",
             batch, heads, keys, need, kNoAllocScratchBytes);
    return omni::set_last_error(OMNIASR_ERR_WORKSPACE, msg);
  }
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices)
    return omni::set_last_error(OMNIASR_ERR_DEVICE, "decode_attention_noalloc: no usable current device");
  cudaError_t err = cudaSuccess;
  void* scratch = scratch_address(device, &err);
  if (!scratch) {
    char msg[256];
    snprintf(msg, sizeof msg, "decode_attention_noalloc: scratch address lookup failed: %s", cudaGetErrorString(err));
    return omni::set_last_error(OMNIASR_ERR_CUDA, msg);
  }
  return omniasr_decode_attention(q, k_cache, v_cache, cache_rows, cache_len, stride_row, stride_head, stride_pos,
                                  lengths, out, batch, heads, dim, keys, scale, dtype, scratch, kNoAllocScratchBytes,
                                  status, stream);
}
