// Failure-path self-test of the bounded device waits.
//
// Every pipelined kernel of this library waits on mbarriers through
// mbar_wait_for (common.cuh): after a time limit the wait records
// FITQ_ERR_TIMEOUT in the library's device status word, sets the kernel's
// abort flag and returns false, so the kernel unwinds and the context stays
// usable instead of hanging.  This kernel exercises exactly that path without
// any fault: one thread waits on a shared-memory mbarrier that nothing
// completes (count 1, no arrival, no copy in flight) with a short limit.
#include "common.cuh"
#include "kernels.cuh"

namespace fitq {
namespace {

__global__ void __launch_bounds__(32) selftest_wait_kernel(int* status, uint64_t limit_ns,
                                                           unsigned long long* elapsed_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_s;
  if (threadIdx.x != 0) return;
  mbar_init(&bar, 1);
  abort_s = 0;
  fence_mbar_init();
  const uint64_t t0 = globaltimer_ns();
  const bool done = mbar_wait_for(&bar, 0, &abort_s, status, limit_ns);
  const uint64_t t1 = globaltimer_ns();
  if (elapsed_ns) *elapsed_ns = done ? 0ull : static_cast<unsigned long long>(t1 - t0);
}

}  // namespace

int launch_selftest_wait(uint64_t limit_ns, unsigned long long* elapsed_ns, int* status,
                         cudaStream_t st) {
  selftest_wait_kernel<<<1, 32, 0, st>>>(status, limit_ns, elapsed_ns);
  note_launch();
  return launch_result();
}

}  // namespace fitq
