// Self-test of the bounded device wait that every kernel of this library uses (mbar_wait, common.cuh).
//
// A kernel waits on an mbarrier initialised for one arrival that never comes: nothing can complete the phase, so
// the wait must give up after the caller's limit, set the timeout bit of the status word and let the kernel
// return. The GPU context stays usable afterwards. This is how a caller can see, without a fault or a hang, that
// the timeout path of the library's waits works on its GPU.

#include "common.cuh"
#include "omniasr_b200.h"

namespace omni {
int set_last_error(int code, const char* message);  // capi.cu
}

namespace {

__global__ void wait_timeout_kernel(uint64_t limit_ns, int* status, unsigned long long* waited_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  omni::mbar_init(&bar, 1);
  omni::mbar_fence_init();
  const uint64_t t0 = omni::global_ns();
  const bool done = omni::mbar_wait(&bar, 0, limit_ns);  // no thread ever arrives
  if (waited_ns) *waited_ns = omni::global_ns() - t0;
  if (!done) omni::raise_status(status, omni::kStatusTimeout);
}

}  // namespace

extern "C" int omniasr_selftest_wait_timeout(int64_t limit_ns, int* status, unsigned long long* waited_ns,
                                             cudaStream_t stream) {
  if (limit_ns <= 0 || limit_ns > 100000000)  // at most 0.1 s: the test must stay short
    return omni::set_last_error(OMNIASR_ERR_ARGUMENT, "selftest_wait_timeout: limit_ns must be in (0, 1e8]");
  wait_timeout_kernel<<<1, 32, 0, stream>>>((uint64_t)limit_ns, status, waited_ns);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return omni::set_last_error(OMNIASR_ERR_CUDA, cudaGetErrorString(e));
  return omni::set_last_error(OMNIASR_OK, "");
}
