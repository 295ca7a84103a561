// Shared device helpers for the omniASR decoder-attention kernels (sm_100a).
//
// Conventions used by every kernel in this library:
//  * Strides are in elements, the innermost (head_dim) stride is 1.
//  * Every device-side index that comes from a tensor (lengths, positions, cache rows, beam
//    pointers) is bounds-checked; an index outside its tensor skips the access and sets a bit in
//    the caller's status word (never a trap).
//  * Every spin-wait is bounded by wall time (kWaitLimitNs); a wait that gives up sets
//    kStatusTimeout and the kernel returns.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define OMNI_DEV __device__ __forceinline__

namespace omni {

constexpr int kStatusIndex = 1;    // an index read from a tensor was outside its tensor
constexpr int kStatusTimeout = 2;  // a bounded wait gave up
constexpr int kStatusLayout = 4;   // a kernel did not run: its shared memory was not laid out as it requires
constexpr uint64_t kWaitLimitNs = 2000000000ull;

OMNI_DEV void raise_status(int* status, int code) {
  if (status) atomicOr(status, code);
}

OMNI_DEV uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

OMNI_DEV uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------------
// mbarrier + 1-D bulk copy (the TMA engine's untiled form): global -> shared, completion counted
// in bytes on an mbarrier.

OMNI_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

OMNI_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

OMNI_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

OMNI_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

OMNI_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probe: has the phase of `parity` completed?
OMNI_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of `parity` to complete; false after `limit_ns` (kWaitLimitNs unless a self-test asks for
// a shorter limit).
OMNI_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > limit_ns) return false;
  }
  return true;
}

// As mbar_wait, but also gives up (false) once *stop is set -- for a role that waits on another role which may
// have abandoned its work.
OMNI_DEV bool mbar_wait_or(uint64_t* bar, uint32_t parity, const volatile int* stop) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (*stop || global_ns() - t0 > kWaitLimitNs) return false;
  }
  return true;
}

OMNI_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// ---------------------------------------------------------------------------------------------
// Element types. Keys/values move as 16-byte vectors; arithmetic is fp32.

template <typename T>
struct Elem;

template <>
struct Elem<float> {
  static constexpr int kVec = 4;  // elements per 16 bytes
  OMNI_DEV static void unpack(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x);
    f[1] = __uint_as_float(u.y);
    f[2] = __uint_as_float(u.z);
    f[3] = __uint_as_float(u.w);
  }
  OMNI_DEV static float to_float(float x) { return x; }
  OMNI_DEV static float from_float(float x) { return x; }
};

template <>
struct Elem<__nv_bfloat16> {
  static constexpr int kVec = 8;
  OMNI_DEV static void unpack(const uint4& u, float* f) {
    f[0] = __uint_as_float(u.x << 16);
    f[1] = __uint_as_float(u.x & 0xffff0000u);
    f[2] = __uint_as_float(u.y << 16);
    f[3] = __uint_as_float(u.y & 0xffff0000u);
    f[4] = __uint_as_float(u.z << 16);
    f[5] = __uint_as_float(u.z & 0xffff0000u);
    f[6] = __uint_as_float(u.w << 16);
    f[7] = __uint_as_float(u.w & 0xffff0000u);
  }
  OMNI_DEV static float to_float(__nv_bfloat16 x) { return __bfloat162float(x); }
  OMNI_DEV static __nv_bfloat16 from_float(float x) { return __float2bfloat16_rn(x); }
};

// 2^x on the special-function unit (MUFU.EX2); ex2(-inf) = 0.
OMNI_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr float kLog2e = 1.4426950408889634f;

// Launches `kern` as a programmatic dependent of the stream's previous kernel: its blocks may start while that
// kernel drains, and must execute griddepcontrol.wait before reading anything an earlier kernel wrote.
template <typename Kern, typename... Args>
inline cudaError_t launch_dependent(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                    Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

OMNI_DEV void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
OMNI_DEV void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace omni
