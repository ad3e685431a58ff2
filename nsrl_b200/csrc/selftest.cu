// nsrl_selftest_bounded_wait: makes one bounded mbarrier wait run out, on
// purpose, so that the timeout path of every kernel's waits can be tested
// without faulting or hanging a GPU.
//
// The kernels' waits (mbar_wait in common.cuh) give up after a time limit,
// set NSRL_FLAG_WAIT_TIMEOUT in the call's status and return false; the
// kernel then unwinds and later CTAs of the call skip their work
// (timed_out()).  Here one CTA initialises an mbarrier that nothing ever
// arrives on and waits for its first phase with the same loop and a caller's
// short limit.  The kernel must come back, report the wait as failed and find
// the flag set; the host then sees NSRL_CORE_REJECTED from
// nsrl_status_fetch.
#include "common.cuh"
#include "internal.h"

namespace {

__global__ void wait_selftest_kernel(unsigned long long limit_ns, nsrl_device_status* st,
                                     unsigned long long* out) {
  __shared__ uint64_t bar;
  __shared__ unsigned int failed;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);  // expects one arrival; none is made
    fence_barrier_init();
    failed = 0;
  }
  __syncthreads();
  const unsigned long long t0 = global_ns();
  const bool ok = mbar_wait_for(&bar, 0, st, limit_ns);
  if (!ok) atomicAdd(&failed, 1u);
  __syncthreads();
  if (threadIdx.x == 0) {
    out[0] = failed;                    // threads whose wait gave up
    out[1] = timed_out(st) ? 1ull : 0;  // what a later CTA of the call would read
    out[2] = global_ns() - t0;          // nanoseconds the waits took
  }
}

}  // namespace

extern "C" nsrl_status nsrl_selftest_bounded_wait(unsigned long long limit_ns, nsrl_device_status* status,
                                                  unsigned long long* out, void* stream) {
  if (!status || !out || limit_ns == 0 || limit_ns > 1000000000ull) {
    nsrl::set_error("invalid argument: bounded-wait self-test (limit in (0, 1 s])");
    return NSRL_INVALID_SHAPE;
  }
  wait_selftest_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(limit_ns, status, out);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    nsrl::set_error("bounded-wait self-test: %s", cudaGetErrorString(e));
    return NSRL_CUDA_ERROR;
  }
  return NSRL_OK;
}
