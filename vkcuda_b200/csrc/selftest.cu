// selftest.cu - exercises the bounded-wait path of the device pipelines
// without hanging the GPU: one thread waits on an mbarrier that nothing
// arrives on, the wait gives up after `timeout_us`, records kErrSelfTest and
// the kernel returns normally, leaving the context usable.
#include <cuda_runtime.h>
#include <cstdint>

#include "internal.h"
#include "ptx.cuh"

namespace vcb {
namespace {

__global__ void bounded_wait_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // Phase 0 never completes: no thread arrives on the barrier.
    const uint32_t addr = smem_u32(&bar);
    const uint64_t t0 = global_timer_ns();
    bool done = false;
    for (uint32_t spin = 1; !done; ++spin) {
      done = mbar_test_parity(addr, 0);
      if (!done && (spin & 63u) == 0u && global_timer_ns() - t0 > limit_ns) break;
    }
    if (!done) atomicCAS(&vc_dev_error, 0u, static_cast<unsigned int>(kErrSelfTest));
  }
}

}  // namespace

cudaError_t launch_selftest_bounded_wait(unsigned timeout_us, cudaStream_t stream) {
  if (timeout_us == 0 || timeout_us > 2000000u) return cudaErrorInvalidValue;
  bounded_wait_kernel<<<1, 32, 0, stream>>>(static_cast<uint64_t>(timeout_us) * 1000ull);
  return cudaGetLastError();
}

}  // namespace vcb

VCB_DEFINE_ERROR_ACCESSOR(selftest_error)
