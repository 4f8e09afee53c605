// Per-thread asynchronous copies global -> shared (cp.async, 4 / 8 / 16 bytes),
// for kernels that stream rows through a small per-lane ring: each lane
// copies its own slice of a row and reads it back itself, so rows are in
// flight without holding them in registers and no lane waits on another.
#pragma once

#include <cstdint>

namespace gmdn {

template <int BYTES>
__device__ __forceinline__ void cp_async(void* smem, const void* gmem) {
  static_assert(BYTES == 4 || BYTES == 8 || BYTES == 16, "cp.async size");
  asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
               "l"(gmem), "n"(BYTES)
               : "memory");
}
// 16 bytes, cached in L2 only (streamed rows are read once)
__device__ __forceinline__ void cp_async_cg16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                   static_cast<uint32_t>(__cvta_generic_to_shared(smem))),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// Wait until at most N of this thread's committed groups are still pending.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace gmdn
