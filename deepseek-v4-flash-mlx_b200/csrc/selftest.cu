// Self-test of the library's failure path: a bounded mbarrier wait that runs out.
//
// The tcgen05 kernels wait on mbarriers for their bulk copies and MMAs, each wait bounded by
// tc5::WAIT_NS of %globaltimer; when a wait runs out, the kernel records DSV4_ERR_WAIT_TIMEOUT on the
// device error word and returns, so that the context stays usable and the host learns of it through
// dsv4_device_error. This entry point exercises exactly that helper (tc5::bar_wait) on a barrier that
// nothing arrives on: the wait ends after WAIT_NS (1 s), the kernel records the timeout and returns.
// Nothing faults, traps or spins without bound.
#include "common.cuh"
#include "tcgen05.cuh"

namespace dsv4 {
namespace st {

__global__ void wait_timeout_kernel() {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    tc5::bar_init(&bar, 1);  // one expected arrival, which never comes
    tc5::bar_init_fence();
  }
  __syncthreads();
  if (threadIdx.x == 0 && !tc5::bar_wait(&bar, 0)) raise_device_error(DSV4_ERR_WAIT_TIMEOUT);
}

}  // namespace st
DSV4_ERROR_READER(selftest)
}  // namespace dsv4

using namespace dsv4;

extern "C" int dsv4_selftest_wait_timeout(void* stream) {
  st::wait_timeout_kernel<<<1, 32, 0, as_stream(stream)>>>();
  DSV4_LAUNCH_CHECK("wait_timeout_kernel");
  return DSV4_OK;
}
