// dash_selftest.cu -- self-test of the bounded mbarrier wait (no reference
// counterpart).  One thread waits for a phase that never completes; the
// helper every kernel uses must give up after the limit, raise the abort flag
// and record DASH_DEV_TIMEOUT, and the kernel returns normally.
#include "dash_common.cuh"
#include "dash_internal.h"

namespace dash {

__global__ void bounded_wait_selftest_kernel(uint64_t limit_ns, DeviceError* err) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);          // one arrival would complete phase 0; none comes
    abort_flag = 0;
    mbar_init_fence();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, &abort_flag, err, 90, limit_ns);
}

}  // namespace dash

extern "C" int dash_selftest_bounded_wait(uint64_t limit_ns, DashDeviceError* err,
                                          dash_stream_t stream) {
  using namespace dash;
  if (limit_ns < 1000000ull || limit_ns > 1000000000ull)
    return set_error(DASH_ERR_INVALID, "limit_ns %llu not in [1 ms, 1 s]",
                     (unsigned long long)limit_ns);
  if (err == nullptr) return set_error(DASH_ERR_INVALID, "null device error word");
  bounded_wait_selftest_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(limit_ns, err);
  count_launch();
  return check_launch("bounded_wait_selftest_kernel");
}
