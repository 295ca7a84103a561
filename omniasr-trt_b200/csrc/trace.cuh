#pragma once

// Per-tile timeline hook for development builds: -DOMNI_TRACE records clock64() of CTA 0's pipeline events into
// omni_trace[] (read back by a tracing harness, which includes one kernel source). Product builds compile it to
// nothing.
#ifdef OMNI_TRACE
__device__ unsigned long long omni_trace[4096];
#define OMNI_TRACE_AT(slot)                                    \
  do {                                                         \
    if (blockIdx.x == 0 && (slot) < 4096) omni_trace[(slot)] = clock64(); \
  } while (0)
// Start / end (global timer, ns) of every CTA at omni_trace[2048 + 2 * cta].
#define OMNI_TRACE_CTA(which)                                                            \
  do {                                                                                   \
    if (threadIdx.x == 0 && blockIdx.x < 1000) {                                         \
      unsigned long long t_;                                                             \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                            \
      omni_trace[2048 + 2 * blockIdx.x + (which)] = t_;                                 \
    }                                                                                    \
  } while (0)
#else
#define OMNI_TRACE_AT(slot) \
  do {                      \
  } while (0)
#define OMNI_TRACE_CTA(which) \
  do {                        \
  } while (0)
#endif

