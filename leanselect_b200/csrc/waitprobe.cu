// ls_wait_timeout_probe: a test hook for the bounded-wait unwind.
//
// Every kernel of this library that waits on an mbarrier (a TMA copy, an
// MMA, a free ring slot) gives up after a wall-time limit, records
// LS_DEVERR_TIMEOUT in the caller's status word, tells the other warps of
// its CTA through a shared abort flag, lets copies in flight land and
// releases its tensor memory before returning.  The probe exercises that
// path on purpose without a fault: one CTA shaped like the scoring kernel
// allocates tensor memory, its producer lane waits for a ring slot nothing
// frees (limit `timeout_ns`), the other warps wait for data nothing sends
// (twice the limit, so they leave through the abort flag), and the CTA then
// unwinds exactly as the real kernels do.  `done` is set when the kernel
// reached its end.
#include "common.cuh"
#include "launch.h"

namespace ls {
namespace {

__global__ void __launch_bounds__(192, 1) wait_probe_kernel(int32_t* status, int32_t* done,
                                                            uint64_t timeout_ns) {
  __shared__ uint64_t bars[2];
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&tmem_base, 32);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  volatile int* abort = &abort_flag;
  if (warp == 0) {
    if (lane == 0) mbar_wait_for(&bars[0], 0, status, abort, timeout_ns);
  } else {
    mbar_wait_for(&bars[1], 0, status, abort, 2 * timeout_ns);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 32);
  }
  if (threadIdx.x == 0) *done = 1;
}

}  // namespace

cudaError_t launch_wait_probe(int32_t* status, int32_t* done, uint64_t timeout_ns,
                              cudaStream_t stream) {
  wait_probe_kernel<<<1, 192, 0, stream>>>(status, done, timeout_ns);
  return cudaGetLastError();
}

}  // namespace ls
