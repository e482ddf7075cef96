// th_selftest_bounded_wait: exercises the bounded mbarrier wait that every
// pipelined kernel of this library uses (mbar_wait_for in common.cuh), with
// a short limit chosen by the caller, so a test can make a wait run out on a
// real GPU without hanging it.
//
// One CTA of 64 threads: thread 0 waits on a shared-memory mbarrier with a
// limit of `limit_ns`; thread 32 arrives on that barrier once `arrive_ns`
// of %globaltimer have passed.  With arrive_ns > limit_ns the wait gives up
// first, sets the device error word (TH_DEVERR_MBAR_TIMEOUT) and writes 0 to
// *completed; otherwise it sees the arrival and writes 1.  The arriver's
// delay is bounded by the host check below, and the CTA drains with a
// __syncthreads after both have finished, so the kernel always ends.
#include "common.cuh"

namespace th {

__global__ void __launch_bounds__(64) selftest_wait_kernel(unsigned long long limit_ns, unsigned long long arrive_ns,
                                                           int* completed) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = mbar_wait_for(&bar, 0, &abort_flag, limit_ns);
    *completed = ok ? 1 : 0;
  } else if (threadIdx.x == 32) {
    const unsigned long long t0 = globaltimer_ns();
    while (globaltimer_ns() - t0 < arrive_ns) {
    }
    mbar_arrive(&bar);
  }
  __syncthreads();
}

}  // namespace th

extern "C" int th_selftest_bounded_wait(int64_t limit_ns, int64_t arrive_ns, int32_t* completed, void* stream) {
  using namespace th;
  if (!completed) return fail(TH_EINVAL, "th_selftest_bounded_wait: completed is NULL");
  // both delays stay far below the library's own 2 s wait limit
  if (limit_ns < 1000 || limit_ns > 100000000 || arrive_ns < 0 || arrive_ns > 100000000)
    return fail(TH_EINVAL, "th_selftest_bounded_wait: limit_ns must be in [1e3, 1e8] and arrive_ns in [0, 1e8]");
  selftest_wait_kernel<<<1, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      (unsigned long long)limit_ns, (unsigned long long)arrive_ns, completed);
  return check_launch("th_selftest_bounded_wait");
}
