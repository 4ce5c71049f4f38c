// selftest.cu -- exercises the timeout path of the bounded mbarrier wait.
//
// Every kernel of this library waits on mbarriers through mbar_wait_ns
// (sm100.cuh): a wait that does not complete within its limit records
// THM_ERR_TIMEOUT in a device status word and returns false, and the kernel
// unwinds instead of spinning forever. In the real kernels nothing makes a
// wait run out, so this translation unit provides one that always does: one
// warp initialises an mbarrier that nobody ever arrives on and waits on it with
// a short limit. Nothing asynchronous (TMA, tcgen05) is in flight, so the kernel
// simply returns once the limit has passed; the host then reads the status
// through thm_get_device_status(), exactly as it would after a real timeout.
#include "host_util.h"
#include "sm100.cuh"

THM_DEFINE_STATUS(g_status_selftest)

namespace thm {
namespace selftest {

__global__ void wait_never_arrives_kernel(uint64_t limit_ns, int* waited_out) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  __syncwarp();
  bool ok = true;
  if (threadIdx.x == 0) {
    ok = mbar_wait_ns(&bar, 0, &g_status_selftest, limit_ns);
    if (waited_out != nullptr) *waited_out = ok ? 0 : 1;
  }
  __syncwarp();
}

}  // namespace selftest
}  // namespace thm

THM_STATUS_READER(thm_internal_status_selftest, g_status_selftest)

extern "C" int thm_selftest_wait_timeout(long long limit_ns, int* waited_out, thm_stream_t stream) {
  // 1 us .. 100 ms: long enough to be a real wait, short enough for a test.
  if (limit_ns < 1000 || limit_ns > 100ll * 1000 * 1000) return THM_ERR_INVALID;
  thm::selftest::wait_never_arrives_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      (uint64_t)limit_ns, waited_out);
  return thm::check_launch();
}
