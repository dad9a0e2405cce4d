// Test-only entry points, compiled only into a build with -DLIFB_TEST_HOOKS
// (the test of the timeout path builds such a library beside the product one;
// the product library exports none of this).
#ifdef LIFB_TEST_HOOKS
#include "lifb_internal.h"
#include "tma.cuh"

namespace lifb {

// One warp waits on phase 0 of an mbarrier that nothing will ever arrive at,
// with no copy issued: the bounded wait expires after kWaitCycles, the kernel
// records kStatusTmaWaitTimeout in the status word and returns, exactly as a
// kernel whose TMA copy never completed would.
__global__ void k_test_stalled_wait(int *status)
{
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncwarp();
    const bool ok = mbar_wait(&bar, 0);
    if (!ok && threadIdx.x == 0 && status) atomicCAS(status, 0, (int)kStatusTmaWaitTimeout);
}

}  // namespace lifb

extern "C" int lifb_test_stalled_wait(void *stream)
{
    lifb::count_launches(1);
    lifb::k_test_stalled_wait<<<1, 32, 0, (cudaStream_t)stream>>>(lifb::device_status_ptr());
    return cudaGetLastError() == cudaSuccess ? LIFB_OK : LIFB_ERR_CUDA;
}
#endif
