// Input gradient of a dense layer on the 5th-generation tensor cores:
// dX [R, Din] = dY [R, Dout] . W [Dout, Din], to fp32 accuracy.
//
// This is the backward of the consumer network's Linear layers
// (lifscan/shdnet.py:30-50: fc(x) feeding a LIF layer; torch computes the
// input gradient as one fp32 GEMM).  The product is done as three TF32 MMAs
// ("3xTF32"): with a = a_hi + a_lo and b = b_hi + b_lo split at the TF32
// mantissa, a*b ~= a_hi*b_hi + a_hi*b_lo + a_lo*b_hi, accumulated in fp32 in
// tensor memory; the dropped a_lo*b_lo term and the rounding of the low parts
// are about 2^-22 relative, so the result agrees with an fp32 GEMM to about
// 1e-6 (not bit for bit: the accumulation order differs).
//
// Layout: one CTA per 128 rows of dY (the MMA's M), all Din columns (N <= 256)
// in one TMEM accumulator of 128 lanes x N fp32 columns.  K = Dout runs in
// chunks of 16 (one 64-byte swizzle row): TMA brings the dY chunk and the
// chunks of W^T's high and low parts (prepared once per call by k_split_wt)
// into a 2-stage ring in the 64-byte swizzled K-major layout; the CTA's 128
// worker threads split the dY chunk in place (high part) and beside it (low
// part); one of them issues the 6 MMAs of the chunk (3 products x 2 MMAs of
// K = 8) and commits them to the stage's barrier, on which a producer warp
// waits to refill the stage while the workers go on to the next one.
// The 48-KB stages let two CTAs share an SM (and its 512 TMEM columns), so
// one CTA's epilogue and waits overlap the other's MMAs.  The epilogue reads
// the accumulator with tcgen05.ld (one row per thread), writes it to shared
// memory in the 128-byte swizzled layout and stores it with TMA, 32 columns
// at a time, four column groups per round.  Every barrier wait is bounded
// (status 101).
#include "lifb_common.cuh"
#include "lifb_internal.h"
#include "tma.cuh"

namespace lifb {

namespace {

constexpr int kDgM = 128;        // rows of dY per CTA (the MMA's M)
constexpr int kDgK = 16;         // K per stage: one 64-byte swizzle row of fp32
constexpr int kDgOutCols = 32;   // columns per output tile: one 128-byte swizzle row
constexpr int kDgOutRound = 4;   // output tiles staged per round (64 KB)
constexpr int kDgStages = 2;
constexpr int kDgThreads = 128;  // worker warps: one TMEM lane quarter each (plus a producer warp)

// Shared-memory matrix descriptor of a K-major operand in the 64-byte
// swizzled layout: rows of 64 bytes, groups of 8 rows 512 bytes apart (stride
// byte offset), leading byte offset unused (1), descriptor version 1, layout
// type 4 (64-byte swizzle).  The tile base must be 512-byte aligned; the K
// steps inside the swizzle row advance the start address by 32 bytes.
__device__ __forceinline__ uint64_t umma_desc_sw64(uint32_t saddr)
{
    return (uint64_t)((saddr & 0x3FFFF) >> 4) | (1ull << 16) | (32ull << 32) | (1ull << 46) | (4ull << 61);
}

// Instruction descriptor of kind::tf32: D fp32 (bits 4-5 = 1), A and B TF32
// (bits 7-9, 10-12 = 2), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__host__ __device__ constexpr uint32_t umma_idesc_tf32(int m, int n)
{
    return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_tf32(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc)
{
    const uint32_t z = 0;  // no output lanes disabled
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %5, %5, %5}, p;\n\t}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(z)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t *bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// The value rounded to TF32 (10 mantissa bits, to nearest), as a 32-bit word
// with the low 13 bits clear.  Rounding, not truncation: truncated parts are
// biased toward zero and their errors add up along K.
__device__ __forceinline__ float tf32_hi(float a)
{
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(a));
    return __uint_as_float(r);
}

}  // namespace

// Wt_hi[n][k], Wt_lo[n][k] from W[k][n] (k < K = Dout, n < N = Din): the
// transposed weight split into its TF32 high part and the TF32 part of the rest,
// rows of Kp >= K (zeros past K, so a last K chunk that reaches past Dout adds
// nothing).
__global__ void k_split_wt(const float *__restrict__ W, float *__restrict__ hi, float *__restrict__ lo, int K, int Kp,
                           int N)
{
    __shared__ float t[32][33];
    const int k0 = blockIdx.y * 32, n0 = blockIdx.x * 32;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int k = k0 + r, n = n0 + threadIdx.x;
        t[r][threadIdx.x] = (k < K && n < N) ? W[(int64_t)k * N + n] : 0.0f;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const int n = n0 + r, k = k0 + threadIdx.x;
        if (n < N && k < Kp) {
            const float a = t[threadIdx.x][r];  // 0 past K
            const float h = tf32_hi(a);
            hi[(int64_t)n * Kp + k] = h;
            lo[(int64_t)n * Kp + k] = tf32_hi(a - h);
        }
    }
}

// dX = dY . W for one 128-row tile per CTA; N = Din (64, 128 or 256), K = Dout
// rounded up to a multiple of 16 (the dY columns past Dout load as zeros);
// tmem_cols: N rounded up to a power of two >= 32.
template <int N>
__global__ void __launch_bounds__(kDgThreads + 32, 2)
    k_dgrad_3xtf32(const __grid_constant__ CUtensorMap tA, const __grid_constant__ CUtensorMap tBh,
                   const __grid_constant__ CUtensorMap tBl, const __grid_constant__ CUtensorMap tC, int K,
                   int *status)
{
    constexpr uint32_t kABytes = kDgM * kDgK * 4;  // 8 KB
    constexpr uint32_t kOutBytes = kDgM * kDgOutCols * 4;  // 16 KB
    constexpr uint32_t kBBytes = N * kDgK * 4;
    constexpr uint32_t kStage = 2 * kABytes + 2 * kBBytes;
    constexpr int kTmemCols = N <= 32 ? 32 : N <= 64 ? 64 : N <= 128 ? 128 : 256;
    constexpr uint32_t kIdesc = umma_idesc_tf32(kDgM, N);
    extern __shared__ unsigned char dg_raw[];
    // 1024-byte alignment of every tile (the largest swizzle atom)
    unsigned char *base = (unsigned char *)(((uintptr_t)dg_raw + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full[kDgStages], done[kDgStages];
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5;
    const int nk = K / kDgK;
    const int m0 = blockIdx.x * kDgM;
    // warps 0-3: split, MMA issue (thread 0), epilogue (TMEM lane quarter = warp);
    // warp 4: the producer, which refills a stage as soon as the MMAs that read it retire
    auto workers_sync = [] { asm volatile("bar.sync 1, %0;" ::"n"(kDgThreads) : "memory"); };

    auto A = [&](int s) { return base + (size_t)s * kStage; };
    auto Alo = [&](int s) { return base + (size_t)s * kStage + kABytes; };
    auto Bh = [&](int s) { return base + (size_t)s * kStage + 2 * kABytes; };
    auto Bl = [&](int s) { return base + (size_t)s * kStage + 2 * kABytes + kBBytes; };

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int s = 0; s < kDgStages; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&done[s], 1);
        }
        abort_flag = 0;
        fence_barrier_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == kDgThreads / 32) {
        if ((tid & 31) == 0) {
            prefetch_tmap(&tA);
            prefetch_tmap(&tBh);
            prefetch_tmap(&tBl);
            for (int c = 0; c < nk; c++) {
                const int s = c % kDgStages;
                // chunk c - kDgStages's MMAs have read the stage
                if (c >= kDgStages && !mbar_wait(&done[s], (uint32_t)((c - kDgStages) / kDgStages) & 1)) {
                    atomicExch(&abort_flag, 1);
                    break;
                }
                if (abort_flag) break;
                mbar_arrive_expect_tx(&full[s], kStage - kABytes);  // A, Bh, Bl (Alo is written by the workers)
                tma_load_2d(A(s), &tA, c * kDgK, m0, &full[s]);
                tma_load_2d(Bh(s), &tBh, c * kDgK, 0, &full[s]);
                tma_load_2d(Bl(s), &tBl, c * kDgK, 0, &full[s]);
            }
        }
    } else {
        int issued = 0;
        for (int c = 0; c < nk; c++) {
            const int s = c % kDgStages;
            const uint32_t ph = (uint32_t)(c / kDgStages) & 1;
            if (!mbar_wait(&full[s], ph)) atomicExch(&abort_flag, 1);
            workers_sync();
            if (abort_flag) break;
            // split the dY chunk: high part in place, low part beside it (same layout)
            float4 *a4 = reinterpret_cast<float4 *>(A(s));
            float4 *l4 = reinterpret_cast<float4 *>(Alo(s));
#pragma unroll
            for (int i = tid; i < (int)(kABytes / 16); i += kDgThreads) {
                float4 v = a4[i], h, l;
                h.x = tf32_hi(v.x); h.y = tf32_hi(v.y); h.z = tf32_hi(v.z); h.w = tf32_hi(v.w);
                l.x = tf32_hi(v.x - h.x); l.y = tf32_hi(v.y - h.y); l.z = tf32_hi(v.z - h.z); l.w = tf32_hi(v.w - h.w);
                a4[i] = h;
                l4[i] = l;
            }
            fence_proxy_async_shared();  // the workers' writes, seen by the tensor cores
            workers_sync();
            if (tid == 0) {
                tc_fence_after();
                const uint32_t sa = smem_u32(A(s)), sl = smem_u32(Alo(s)), sh = smem_u32(Bh(s)), sb = smem_u32(Bl(s));
#pragma unroll
                for (int kk = 0; kk < kDgK / 8; kk++) {
                    const uint32_t off = kk * 32;  // 8 tf32 = 32 bytes along K inside the swizzle row
                    const uint64_t da = umma_desc_sw64(sa + off), dl = umma_desc_sw64(sl + off);
                    const uint64_t dh = umma_desc_sw64(sh + off), db = umma_desc_sw64(sb + off);
                    umma_tf32(tmem, da, dh, kIdesc, (c > 0 || kk > 0) ? 1u : 0u);
                    umma_tf32(tmem, da, db, kIdesc, 1u);
                    umma_tf32(tmem, dl, dh, kIdesc, 1u);
                }
                umma_commit(&done[s]);
            }
            issued = c + 1;
        }
        workers_sync();
        // the last commit tracks every MMA issued before it
        if (issued > 0 && !mbar_wait(&done[(issued - 1) % kDgStages], (uint32_t)((issued - 1) / kDgStages) & 1))
            atomicExch(&abort_flag, 1);
        workers_sync();  // one decision for all workers
        const bool ok = !abort_flag && issued == nk;
        if (!ok && tid == 0) atomicExch(status, kStatusTmaWaitTimeout);
        tc_fence_after();
        if (ok) {
            // epilogue: TMEM -> registers -> swizzled smem -> TMA store, 32 columns
            // per tile, kDgOutRound tiles per round
            const int row = warp * 32 + (tid & 31);
            const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
#pragma unroll 1
            for (int g0 = 0; g0 < N / kDgOutCols; g0 += kDgOutRound) {
#pragma unroll 1
                for (int g = g0; g < g0 + kDgOutRound && g < N / kDgOutCols; g++) {
                    uint32_t r[32];
                    tmem_ld32(tmem + lane_base + (uint32_t)(g * kDgOutCols), r);
                    unsigned char *tile = base + (size_t)(g - g0) * kOutBytes;  // [128 rows][128 bytes], swizzled
                    uint4 *rowp = reinterpret_cast<uint4 *>(tile + row * 128);
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        rowp[j ^ (row & 7)] = make_uint4(r[4 * j], r[4 * j + 1], r[4 * j + 2], r[4 * j + 3]);
                }
                fence_proxy_async_shared();
                workers_sync();
                if (tid == 0) {
                    for (int g = g0; g < g0 + kDgOutRound && g < N / kDgOutCols; g++)
                        tma_store_2d(&tC, g * kDgOutCols, m0, base + (size_t)(g - g0) * kOutBytes);
                    bulk_commit();
                    bulk_wait_all();  // the staging tiles are reused by the next round
                }
                workers_sync();
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
    }
}

static int64_t padded_k(int64_t Dout) { return (Dout + kDgK - 1) / kDgK * kDgK; }

size_t dgrad_tc_workspace_bytes(int64_t Din, int64_t Dout) { return (size_t)2 * Din * padded_k(Dout) * 4; }

bool dgrad_tc_applies(int64_t R, int64_t Din, int64_t Dout)
{
    return R > 0 && Dout > 0 && Dout % 4 == 0 && (Din == 64 || Din == 128 || Din == 256) &&
           R < (int64_t(1) << 31);
}

template <int N>
static bool launch_dgrad(const float *dY, const float *Wt_hi, const float *Wt_lo, float *dX, int64_t R, int64_t K,
                         int64_t Kp, cudaStream_t s)
{
    CUtensorMap mA, mBh, mBl, mC;
    if (!make_tmap_2d_swz(&mA, dY, K, R, kDgM, kDgK * 4) || !make_tmap_2d_swz(&mBh, Wt_hi, Kp, N, N, kDgK * 4) ||
        !make_tmap_2d_swz(&mBl, Wt_lo, Kp, N, N, kDgK * 4) || !make_tmap_2d_swz(&mC, dX, N, R, kDgM, kDgOutCols * 4))
        return false;
    constexpr size_t stage = (size_t)2 * kDgM * kDgK * 4 + (size_t)2 * N * kDgK * 4;
    constexpr int rounds_tiles = N / kDgOutCols < kDgOutRound ? N / kDgOutCols : kDgOutRound;
    const size_t epi = (size_t)rounds_tiles * kDgM * kDgOutCols * 4;
    const size_t smem = (kDgStages * stage > epi ? kDgStages * stage : epi) + 1024;
    auto kern = k_dgrad_3xtf32<N>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return false;
    count_launches(1);
    kern<<<(unsigned)((R + kDgM - 1) / kDgM), kDgThreads + 32, smem, s>>>(mA, mBh, mBl, mC, (int)Kp,
                                                                        device_status_ptr());
    return true;
}

bool dgrad_tc(const float *dY, const float *W, float *dX, int64_t R, int64_t Din, int64_t Dout, void *ws,
              cudaStream_t s)
{
    if (!dgrad_tc_applies(R, Din, Dout)) return false;
    const void *p[] = {dY, W, dX, ws};
    for (const void *q : p)
        if (((uintptr_t)q & 15)) return false;
    const int64_t Kp = padded_k(Dout);
    float *hi = (float *)ws, *lo = hi + Din * Kp;
    count_launches(1);
    k_split_wt<<<dim3((unsigned)((Din + 31) / 32), (unsigned)((Kp + 31) / 32)), dim3(32, 8), 0, s>>>(
        W, hi, lo, (int)Dout, (int)Kp, (int)Din);
    if (Din == 256) return launch_dgrad<256>(dY, hi, lo, dX, R, Dout, Kp, s);
    if (Din == 128) return launch_dgrad<128>(dY, hi, lo, dX, R, Dout, Kp, s);
    return launch_dgrad<64>(dY, hi, lo, dX, R, Dout, Kp, s);
}

}  // namespace lifb

extern "C" size_t lifb_dense_dgrad_workspace_bytes(int64_t Din, int64_t Dout)
{
    return lifb::dgrad_tc_workspace_bytes(Din, Dout);
}

extern "C" int lifb_dense_dgrad(const float *dY, const float *W, float *dX, int64_t R, int64_t Din, int64_t Dout,
                                void *workspace, size_t workspace_bytes, void *stream)
{
    LIFB_RANGE("lifb_dense_dgrad");
    if (R < 0 || Din < 0 || Dout < 0) {
        lifb::set_last_error("lifb_dense_dgrad: negative shape");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (R == 0 || Din == 0) return LIFB_OK;
    if (!dY || !W || !dX || !workspace) {
        lifb::set_last_error("lifb_dense_dgrad: null pointer");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (workspace_bytes < lifb::dgrad_tc_workspace_bytes(Din, Dout)) {
        lifb::set_last_error("lifb_dense_dgrad: workspace too small");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (!lifb::dgrad_tc_applies(R, Din, Dout)) {
        lifb::set_last_error("lifb_dense_dgrad: needs Dout % 4 == 0 and Din in {64, 128, 256}");
        return LIFB_ERR_UNSUPPORTED;
    }
    if (!lifb::dgrad_tc(dY, W, dX, R, Din, Dout, workspace, (cudaStream_t)stream)) {
        lifb::set_last_error("lifb_dense_dgrad: pointers must be 16-byte aligned");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (cudaGetLastError() != cudaSuccess) {
        lifb::set_last_error("lifb_dense_dgrad: launch failed");
        return LIFB_ERR_CUDA;
    }
    lifb::set_last_error("");
    return LIFB_OK;
}
