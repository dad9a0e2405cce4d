// Host runtime pieces shared by the kernels: TMA tensor-map encoding through
// the driver entry point (no link-time libcuda dependency) and the per-device
// status word that bounded device-side waits write into.
#include <mutex>

#include <cudaTypedefs.h>

#include "lifb_internal.h"

namespace lifb {

// One status word per device: 0 = ok, else the first device-side error code
// (a bounded wait that expired).  Kernels receive its address as a parameter.
__device__ int g_status_word = 0;

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
constexpr int kMaxDevices = 64;
int *g_status_ptr[kMaxDevices] = {};
std::mutex g_status_mu;
}  // namespace

static PFN_cuTensorMapEncodeTiled_v12000 encoder()
{
    std::call_once(g_encode_once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = (PFN_cuTensorMapEncodeTiled_v12000)fn;
    });
    return g_encode;
}

bool make_tmap_2d(CUtensorMap *m, const float *base, int64_t N, int64_t T, int box_x, int box_y)
{
    return make_tmap_2d_typed(m, base, false, N, T, box_x, box_y);
}

// The encoder is a driver-API call and needs the device's primary context
// current on the calling thread.  A thread whose first CUDA work is this call
// (autograd's backward worker, say, when every allocation it makes is served
// from the caching allocator) has none bound yet: bind it once per device.
static void bind_primary_context()
{
    thread_local int bound = -1;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev != bound && cudaSetDevice(dev) == cudaSuccess) bound = dev;
}

bool make_tmap_2d_typed(CUtensorMap *m, const void *base, bool int32, int64_t N, int64_t T, int box_x, int box_y)
{
    bind_primary_context();
    auto enc = encoder();
    if (!enc || ((uintptr_t)base & 15) || (N * 4) % 16 || T >= (int64_t(1) << 31) || N >= (int64_t(1) << 31))
        return false;
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)T};
    cuuint64_t strides[1] = {(cuuint64_t)N * 4};
    cuuint32_t box[2] = {(cuuint32_t)box_x, (cuuint32_t)box_y};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, int32 ? CU_TENSOR_MAP_DATA_TYPE_INT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base,
                     dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tmap_2d_swz(CUtensorMap *m, const float *base, int64_t N, int64_t T, int box_y, int swz_bytes)
{
    bind_primary_context();
    auto enc = encoder();
    if (!enc || ((uintptr_t)base & 15) || (N * 4) % 16 || T >= (int64_t(1) << 31) || N >= (int64_t(1) << 31) ||
        box_y < 1 || box_y > 256 || (swz_bytes != 64 && swz_bytes != 128))
        return false;
    cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)T};
    cuuint64_t strides[1] = {(cuuint64_t)N * 4};
    cuuint32_t box[2] = {(cuuint32_t)(swz_bytes / 4), (cuuint32_t)box_y};  // one swizzle row of floats
    cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void *)base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE,
                     swz_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool make_tmap_3d_u32(CUtensorMap *m, const void *base, int64_t d0, int64_t d1, int64_t d2, int b0, int b1, int b2)
{
    bind_primary_context();
    auto enc = encoder();
    if (!enc || ((uintptr_t)base & 15) || (d0 * 4) % 16 || d0 >= (int64_t(1) << 31) || d1 >= (int64_t(1) << 31) ||
        d2 >= (int64_t(1) << 31) || b0 > 256 || b1 > 256 || b2 > 256)
        return false;
    cuuint64_t dims[3] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2};
    cuuint64_t strides[2] = {(cuuint64_t)d0 * 4, (cuuint64_t)(d0 * d1) * 4};
    cuuint32_t box[3] = {(cuuint32_t)b0, (cuuint32_t)b1, (cuuint32_t)b2};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_INT32, 3, (void *)base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

int *device_status_ptr()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
    std::lock_guard<std::mutex> g(g_status_mu);
    if (!g_status_ptr[dev]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
        g_status_ptr[dev] = (int *)p;
    }
    return g_status_ptr[dev];
}

// Asynchronous reads of the status word, per device: a pinned host mirror
// filled by a copy on a private non-blocking stream, and an event marking
// when the copy has landed.
namespace {
struct StatusPoll {
    int *mirror = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t landed = nullptr;
    bool pending = false;
    int last = 0;  // the word as of the last completed read
};
StatusPoll g_poll[kMaxDevices];
}  // namespace

int read_device_status(bool reset)
{
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_status_word, sizeof(int)) != cudaSuccess) return -1;
    if (reset && v) {
        int z = 0;
        cudaMemcpyToSymbol(g_status_word, &z, sizeof(int));
        int dev = 0;
        if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kMaxDevices) {
            // a read still in flight may have seen the old value
            std::lock_guard<std::mutex> g(g_status_mu);
            StatusPoll &p = g_poll[dev];
            if (p.pending) cudaStreamSynchronize(p.stream);
            p.pending = false;
            p.last = 0;
        }
    }
    return v;
}

int poll_device_status()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return -1;
    std::lock_guard<std::mutex> g(g_status_mu);
    StatusPoll &p = g_poll[dev];
    if (!p.mirror) {
        if (cudaHostAlloc((void **)&p.mirror, sizeof(int), cudaHostAllocDefault) != cudaSuccess) {
            p.mirror = nullptr;
            return -1;
        }
        *p.mirror = 0;
        if (cudaStreamCreateWithFlags(&p.stream, cudaStreamNonBlocking) != cudaSuccess ||
            cudaEventCreateWithFlags(&p.landed, cudaEventDisableTiming) != cudaSuccess)
            return -1;
    }
    if (p.pending) {
        const cudaError_t q = cudaEventQuery(p.landed);
        if (q == cudaSuccess) {
            p.last = *(volatile int *)p.mirror;
            p.pending = false;
        } else if (q != cudaErrorNotReady) {
            return -1;
        }
    }
    if (!p.pending) {
        if (cudaMemcpyFromSymbolAsync(p.mirror, g_status_word, sizeof(int), 0, cudaMemcpyDeviceToHost, p.stream) !=
                cudaSuccess ||
            cudaEventRecord(p.landed, p.stream) != cudaSuccess)
            return -1;
        p.pending = true;
    }
    return p.last;
}

}  // namespace lifb
