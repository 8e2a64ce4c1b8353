// Self-test of the bounded waits that every tensor-core kernel of this library
// relies on (wait_phase in bm_tc.cuh). One CTA waits on an mbarrier that nothing
// ever completes, with a short limit: the wait must give up, OR
// BM_DEVERR_TIMEOUT into the status word and let the kernel finish, so that the
// CUDA context stays usable. A second thread then waits on the same barrier
// honouring the abort flag the first one set, and must give up at once. No
// fault, trap or endless loop is involved: the failure is a barrier nobody
// arrives at, and every wait is bounded by time and by a poll count.
#include "bm_host.h"
#include "bm_tc.cuh"

namespace bm {
namespace {

// result[0] / [2]: 1 if the first / second wait reported success (expected 0);
// result[1] / [3]: their durations in ns.
__global__ void __launch_bounds__(64) bounded_wait_selftest_kernel(int32_t* status, uint64_t limit_ns,
                                                                   int64_t* result) {
  grid_dependency_wait();
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);  // one arrival would complete it; none comes
    abort_flag = 0;
    tc::fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint64_t t0 = tc::global_ns();
    const bool ok = tc::wait_phase(&bar, 0, &abort_flag, status, limit_ns, false);
    result[0] = ok ? 1 : 0;
    result[1] = static_cast<int64_t>(tc::global_ns() - t0);
  }
  __syncthreads();
  if (threadIdx.x == 32) {
    const uint64_t t0 = tc::global_ns();
    const bool ok = tc::wait_phase(&bar, 0, &abort_flag, status, 100 * limit_ns, true);
    result[2] = ok ? 1 : 0;
    result[3] = static_cast<int64_t>(tc::global_ns() - t0);
  }
}

}  // namespace
}  // namespace bm

extern "C" int bm_selftest_bounded_wait(int64_t limit_ns, int32_t* d_status, int64_t* d_result, void* stream) {
  using namespace bm;
  const char* what = "bm_selftest_bounded_wait";
  if (!d_status || !d_result) return fail(BM_ERR_INVALID_ARGUMENT, "%s: NULL pointer", what);
  if (limit_ns < 1000000 || limit_ns > 2000000000) {
    return fail(BM_ERR_INVALID_ARGUMENT, "%s: limit_ns outside [1 ms, 2 s]", what);
  }
  if (const int launch_status = launch_kernel("bounded_wait_selftest_kernel", bounded_wait_selftest_kernel, dim3(1),
                                              dim3(64), 0, as_stream(stream), nullptr, d_status,
                                              static_cast<uint64_t>(limit_ns), d_result)) {
    return launch_status;
  }
  return check_launch(what);
}
