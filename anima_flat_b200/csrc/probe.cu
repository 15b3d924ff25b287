// Failure-path probe of the bounded waits (no reference counterpart).
//
// Every kernel of this library waits on its bulk copies through mbar_wait,
// which gives up after a bounded number of try_wait rounds, sets the device
// status word and lets the kernel drain its copies in flight and return
// (afb_device.cuh).  In the kernels proper that branch only runs if a copy
// never lands.  This probe takes the same branch on purpose, without any
// fault: one thread starts a real 1 KiB bulk copy on one mbarrier, then waits
// with a short limit on a second mbarrier that nothing ever arrives on, so
// the wait gives up; it then drains the first copy with the normal bounded
// wait and returns.  result[0] = 1 when the unfinished wait gave up,
// result[1] = 1 when the copy in flight was drained.
#include "afb_device.cuh"
#include "afb_launch.h"

namespace afb {

constexpr uint32_t kProbeBytes = 1024;
static __device__ __align__(16) uint8_t g_probe_src[kProbeBytes];

__global__ void __launch_bounds__(32) wait_probe_kernel(uint32_t spins, int* result) {
  __shared__ __align__(128) uint8_t buf[kProbeBytes];
  __shared__ __align__(8) uint64_t bars[2];
  if (threadIdx.x != 0) return;
  const uint32_t copy_bar = smem_addr(&bars[0]);
  const uint32_t never_bar = smem_addr(&bars[1]);
  mbar_init(copy_bar, 1);
  mbar_init(never_bar, 1);
  fence_mbar_init();
  mbar_arrive_expect_tx(copy_bar, kProbeBytes);
  bulk_g2s(smem_addr(buf), g_probe_src, kProbeBytes, copy_bar);
  const bool gave_up = !mbar_wait(never_bar, 0, spins);  // nothing arrives: bounded give-up
  const bool drained = mbar_wait(copy_bar, 0);             // the copy in flight completes
  result[0] = gave_up ? 1 : 0;
  result[1] = drained ? 1 : 0;
}

cudaError_t read_status_probe(int* status, bool clear) { return tu_status(status, clear); }

}  // namespace afb

using namespace afb;

extern "C" int afb_wait_probe(uint32_t spins, void* result, void* stream) {
  ApiGuard g("afb_wait_probe");
  if (!check(spins >= 1 && spins <= (1u << 16), "spins must be in [1, 65536]") ||
      !check_ptr4(result, "result"))
    return g.fail();
  wait_probe_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(spins, static_cast<int*>(result));
  return g.done(cudaGetLastError());
}
