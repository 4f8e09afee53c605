// Failure-detection self-test: one CTA waits, with the kernels' own bounded
// wait (tc.cuh mbar_wait_for, here with a caller-chosen limit), on an mbarrier
// that nothing ever arrives on.  The wait gives up, raises the CTA's abort
// flag (so the second warp leaves too), ORs kStatusWaitTimeout into the
// status word and the kernel returns -- no trap, no fault, the context stays
// usable.  Tests read the word and then run an ordinary op on the same context.

#include <cuda_runtime.h>

#include "fast_path.h"
#include "tc.cuh"

namespace gmdn {
namespace {

__global__ void __launch_bounds__(64, 1) wait_timeout_selftest_kernel(uint32_t* status,
                                                                       uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);   // one arrival expected; none is ever made
    abort_flag = 0;
    tc::fence_mbar_init();
  }
  __syncthreads();
  // every lane of both warps waits, warp-uniformly as the kernels' warp roles do
  const bool ok = __all_sync(0xffffffffu,
                             tc::mbar_wait_for(&bar, 0, status, &abort_flag, limit_ns));
  if (ok && threadIdx.x == 0) atomicOr(status, 0x80000000u);   // must not happen
  __syncthreads();
}

}  // namespace

cudaError_t wait_timeout_selftest(uint32_t* status, uint64_t limit_ns, cudaStream_t st) {
  wait_timeout_selftest_kernel<<<1, 64, 0, st>>>(status, limit_ns);
  return cudaGetLastError();
}

}  // namespace gmdn
