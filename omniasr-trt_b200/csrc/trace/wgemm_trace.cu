// Development build of the decode GEMM with a per-CTA timeline (built by `make -C omniasr-trt_b200/csrc trace` into
// lib/libomniasr_b200_trace.so; read by wgemm_timeline.py). wgemm.cu's OMNI_WG_EVENT hooks store %globaltimer at
// each pipeline event of every CTA, in one slot per GEMM shape of the decoder step (so that one step's four calls,
// run back to back, can be read afterwards); the product build compiles the hooks to nothing.
//
// Events: 0 entry, 1 past the dependency wait, 2 first weight load issued, 3 first stage landed (MMA issuer),
// 4 last MMA issued, 5 last accumulator taken (stream-K epilogue), 6 epilogue done, 7 exit; 9 / 10 / 11 the last
// split tile's watch ended with the other contributors all in / the own accumulator first / a timeout; 12 / 13 a
// tile's write-out started / done (stream-K), 14 arrival counted (stream-K) -- in cluster mode 11 before the cluster
// barrier, 12 after it, 13 the rows summed, 14 written out, 15 past the second barrier.
#include <cstdint>

#include <cuda_runtime.h>

__device__ unsigned long long g_wg_trace[4][256][16];

// The decoder step's four shapes (config 4): QKV 12288 x 4096, output 4096 x 4096, gate/inner 11008 x 4096 (SwiGLU
// outputs), FFN output 4096 x 11008.
__device__ __forceinline__ int wg_trace_slot(int n, int k) {
  return n == 12288 ? 0 : (n == 4096 && k == 4096) ? 1 : n == 11008 ? 2 : 3;
}

#define OMNI_WG_EVENT(a, ev)                                          \
  do {                                                                \
    if (blockIdx.x < 256) {                                           \
      unsigned long long t_;                                          \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));         \
      g_wg_trace[wg_trace_slot((a).n, (a).k)][blockIdx.x][(ev)] = t_; \
    }                                                                 \
  } while (0)

#include "../wgemm.cu"

extern "C" int omni_wg_trace_read(void* dst) {
  return (int)cudaMemcpyFromSymbol(dst, g_wg_trace, sizeof(g_wg_trace));
}

extern "C" int omni_wg_trace_clear() {
  static unsigned long long zeros[4 * 256 * 16];
  return (int)cudaMemcpyToSymbol(g_wg_trace, zeros, sizeof(zeros));
}
