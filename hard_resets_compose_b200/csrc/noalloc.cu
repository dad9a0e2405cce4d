// lifb_scan_fwd_v3_noalloc: the two-level exact scan forward for callers that
// must not allocate device memory when they call into this library.
//
// lifb_scan_fwd_v3 needs a scratch buffer (chunk maps, envelope bounds,
// chunk starts and ends) that its caller allocates.  Some callers cannot do
// that at call time: a plain C or FFI host with no device allocator of its
// own, an application whose whole device-memory budget is already handed to
// another pool or capped by its process limits, or a latency-critical loop
// that must never call cudaMalloc because it can block on the device.  This
// entry point takes only inputs and outputs; its scratch is the fixed array
// below, which every GPU that loads the library holds until the process
// exits.
#include <stdio.h>

#include <mutex>

#include <cudaTypedefs.h>

#include "lifb_internal.h"

namespace {

// The scratch shared by every call of lifb_scan_fwd_v3_noalloc on a device.
static __device__ __align__(256) unsigned char g_noalloc_scratch[LIFB_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
// Device address of g_noalloc_scratch per device, valid for the context it
// was looked up in: a context torn down and made again (cudaDeviceReset)
// reloads the module, and the array may then sit at another address.
void *g_scratch_dev[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

int report(int status, const char *msg)
{
    lifb::set_last_error(msg);
    return status;
}

// The calling thread's current context, through the driver entry point (no
// link-time libcuda dependency); nullptr if it cannot be queried.
CUcontext current_context()
{
    static PFN_cuCtxGetCurrent_v4000 get = [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            fn = nullptr;
        return (PFN_cuCtxGetCurrent_v4000)fn;
    }();
    CUcontext c = nullptr;
    if (!get || get(&c) != CUDA_SUCCESS) return nullptr;
    return c;
}

}  // namespace

extern "C" int lifb_scan_fwd_v3_noalloc(const float *I, const float *u0, float *U, float *S, int64_t T,
                                        int64_t N, float beta, float theta, float u_r, int C, int K,
                                        int max_repair, lifb_stats *stats_dev, void *stream)
{
    LIFB_RANGE("lifb_scan_fwd_v3_noalloc");
    // Size check first: nothing touches the GPU when the request cannot fit.
    const size_t need = lifb_scan_fwd_v3_workspace_bytes(T, N, C, K);
    if (need > (size_t)LIFB_NOALLOC_SCRATCH_BYTES) {
        char buf[256];
        snprintf(buf, sizeof(buf),
                 "lifb_scan_fwd_v3_noalloc: T=%lld N=%lld C=%d K=%d needs %zu bytes of scratch, above the fixed "
                 "%llu-byte no-allocation scratch; use lifb_scan_fwd_v3 with a caller workspace",
                 (long long)T, (long long)N, C, K, need, (unsigned long long)LIFB_NOALLOC_SCRATCH_BYTES);
        return report(LIFB_ERR_INVALID_ARGUMENT, buf);
    }
    // One-time set-up per device, with that device current: the host-side name
    // g_noalloc_scratch is not a device address, so look the address up.
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0)
        return report(LIFB_ERR_CUDA, "lifb_scan_fwd_v3_noalloc: cannot query the current device");
    if (dev >= kMaxDevices) {
        char buf[160];
        snprintf(buf, sizeof(buf), "lifb_scan_fwd_v3_noalloc: device %d is beyond the %d devices this entry point "
                 "serves", dev, kMaxDevices);
        return report(LIFB_ERR_UNSUPPORTED, buf);
    }
    // The first call on a device (and the first in a new context of it) looks
    // the address up; it should come before any stream capture.
    cudaSetDevice(dev);  // binds the device's primary context to this thread if none is
    const CUcontext ctx = current_context();
    void *scratch = nullptr;
    {
        std::lock_guard<std::mutex> g(g_mu);
        if (!g_scratch_dev[dev] || !ctx || g_scratch_ctx[dev] != ctx) {
            void *p = nullptr;
            cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if (e != cudaSuccess || p == nullptr) {
                char buf[256];
                snprintf(buf, sizeof(buf), "lifb_scan_fwd_v3_noalloc: cudaGetSymbolAddress failed: %s",
                         cudaGetErrorString(e));
                return report(LIFB_ERR_CUDA, buf);
            }
            g_scratch_dev[dev] = p;
            g_scratch_ctx[dev] = current_context();  // the context the lookup ran in
        }
        scratch = g_scratch_dev[dev];
    }
    // Every word of scratch the forward reads is written earlier in the same
    // call, so nothing needs clearing between calls.
    return lifb_scan_fwd_v3(I, u0, U, S, T, N, beta, theta, u_r, C, K, max_repair, scratch,
                            (size_t)LIFB_NOALLOC_SCRATCH_BYTES, stats_dev, stream);
}
