// selftest.cu - a failure-detection check that faults nothing: a kernel waits
// on an mbarrier that nothing signals, through the same bounded wait every
// pipeline in this library uses.  The wait gives up after HCU_WAIT_NS of
// %globaltimer, records HCU_DEVERR_TIMEOUT in the handle's device status word
// and returns, so the context stays usable and the host reads the error.
#include "common.cuh"
#include "context.h"

namespace {

using namespace hcu;

__global__ void __launch_bounds__(32) wait_timeout_kernel(uint32_t* status) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncwarp();
  // nothing arrives on `bar`: phase 0 never completes
  (void)mbar_wait(&bar, 0, status);
}

}  // namespace

extern "C" int hcu_selftest_wait_timeout(hcu_handle h) {
  HCU_TRY(hcu::begin_op(h, "hcu_selftest_wait_timeout"));
  wait_timeout_kernel<<<1, 32, 0, h->stream>>>(h->dev_status);
  return hcu::after_launch("hcu_selftest_wait_timeout");
}
