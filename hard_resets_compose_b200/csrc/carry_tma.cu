// Sequential map carry with TMA-staged map windows (carry2_kernel,
// lifscan/triton_lif.py:578-606, evaluated like fast.eval_map, lifscan/fast.py:242-251).
//
// The carry is the one inherently sequential phase of the scan: start_{m+1} =
// map_m(start_m), per neuron.  A warp owns 32 neurons; windows of W maps
// ([M, N] arrays A, B, count, overflow and the [M*K, N] breakpoint and
// constant slabs) arrive in shared memory by TMA, two windows in flight, so a
// hop costs shared-memory latency instead of a global round trip.  All K
// breakpoints of a map are read at once (they do not depend on the state),
// the piece index is the count of breakpoints above the state, and the
// constant is read once the index is known.
//
// Overflowed maps (more than K breakpoints were needed) are still exact for
// states at or above their lowest stored breakpoint, because every dropped
// breakpoint lies below it; there the stored constant equals what the serial
// replay of the map's rows would give.  Only below it does the carry replay
// the rows (L of them) serially from I.
#include "lifb_common.cuh"
#include "lifb_internal.h"
#include "tma.cuh"

namespace lifb {

template <int K, int W>
struct CarryStage {
    // rows of 32 lanes
    static constexpr int kA = 0, kB = W, kN = 2 * W, kO = 3 * W, kX = 4 * W, kC = 4 * W + W * K;
    static constexpr int kRows = 4 * W + 2 * W * K;
    static constexpr uint32_t kBytes = kRows * 32 * 4;
};

template <int K, int W>
__global__ void __launch_bounds__(32) k_carry_staged(const __grid_constant__ CUtensorMap tA,
                                                     const __grid_constant__ CUtensorMap tB,
                                                     const __grid_constant__ CUtensorMap tN,
                                                     const __grid_constant__ CUtensorMap tO,
                                                     const __grid_constant__ CUtensorMap tX,
                                                     const __grid_constant__ CUtensorMap tC,
                                                     const float *__restrict__ I, const float *__restrict__ u0,
                                                     float *__restrict__ Starts, int64_t N, int64_t M, int64_t L,
                                                     float beta, float theta, float u_r, int *status)
{
    using St = CarryStage<K, W>;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    float *buf = reinterpret_cast<float *>(smem_raw);  // 2 stages x kRows x 32
    __shared__ __align__(8) uint64_t full[2];
    const int lane = threadIdx.x;
    const int64_t n0 = (int64_t)blockIdx.x * 32;
    const int64_t n = n0 + lane;
    const bool act = n < N;
    const int64_t nwin = (M + W - 1) / W;

    auto issue = [&](int s, int64_t w) {
        float *b = buf + (size_t)s * St::kRows * 32;
        const int row = (int)(w * W);
        mbar_arrive_expect_tx(&full[s], St::kBytes);
        tma_load_2d(b + St::kA * 32, &tA, (int)n0, row, &full[s]);
        tma_load_2d(b + St::kB * 32, &tB, (int)n0, row, &full[s]);
        tma_load_2d(b + St::kN * 32, &tN, (int)n0, row, &full[s]);
        tma_load_2d(b + St::kO * 32, &tO, (int)n0, row, &full[s]);
        tma_load_2d(b + St::kX * 32, &tX, (int)n0, row * K, &full[s]);
        tma_load_2d(b + St::kC * 32, &tC, (int)n0, row * K, &full[s]);
    };

    if (lane == 0) {
        for (int s = 0; s < 2; s++) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncwarp();
    if (lane == 0) {
        issue(0, 0);
        if (nwin > 1) issue(1, 1);
    }
    float u = act ? u0[n] : 0.0f;
    for (int64_t w = 0; w < nwin; w++) {
        const int s = (int)(w & 1);
        if (!mbar_wait(&full[s], (uint32_t)((w >> 1) & 1))) {
            if (status) atomicCAS(status, 0, (int)kStatusTmaWaitTimeout);
            return;
        }
        const float *b = buf + (size_t)s * St::kRows * 32 + lane;
        const int nm = (int)((M - w * W) < W ? (M - w * W) : W);
        for (int j = 0; j < nm; j++) {
            const int64_t m = w * W + j;
            if (act) Starts[m * N + n] = u;
            if (m + 1 == M) break;  // the last map's value is never used
            const float A = b[(St::kA + j) * 32], B = b[(St::kB + j) * 32];
            const int cnt = __float_as_int(b[(St::kN + j) * 32]);
            const int ovf = __float_as_int(b[(St::kO + j) * 32]);
            float x[K];
#pragma unroll
            for (int i = 0; i < K; i++) x[i] = b[(St::kX + j * K + i) * 32];
            int k = 0;
            float xlast = x[0];
#pragma unroll
            for (int i = 0; i < K; i++) {
                if (i < cnt) {
                    k += x[i] > u ? 1 : 0;  // breakpoints descend: the count is the leading run
                    xlast = x[i];
                }
            }
            float nu;
            if (!ovf || (cnt > 0 && u >= xlast)) {
                nu = (k == cnt) ? mul_add_rn(A, u, B) : b[(St::kC + j * K + k) * 32];
            } else {  // below an overflowed map's stored breakpoints: replay its rows
                float w0 = u;
                const float *p = I + (m * L) * N + n;
                constexpr int kB = 16;  // rows loaded ahead of the dependent steps
                if (act) {
                    for (int64_t r = 0; r < L; r += kB) {
                        float xr[kB];
#pragma unroll
                        for (int q = 0; q < kB; q++) xr[q] = (r + q < L) ? __ldg(p + (r + q) * N) : 0.0f;
#pragma unroll
                        for (int q = 0; q < kB; q++)
                            if (r + q < L) w0 = lif_step_u(w0, xr[q], beta, theta, u_r);
                    }
                }
                nu = w0;
            }
            u = nu;
        }
        __syncwarp();
        if (lane == 0 && w + 2 < nwin) issue(s, w + 2);
    }
}

// Envelope prefix (env_carry_kernel, lifscan/triton_lif.py:722-733) with the
// chunk envelope maps (c, a, b) staged by TMA in windows of W chunks: the same
// arithmetic as k_env_carry, so Lo is identical.
template <int W>
__global__ void __launch_bounds__(32) k_env_carry_staged(const __grid_constant__ CUtensorMap tC,
                                                         const __grid_constant__ CUtensorMap tA,
                                                         const __grid_constant__ CUtensorMap tB,
                                                         const float *__restrict__ u0, float *__restrict__ Lo, int64_t N,
                                                         int64_t M, float margin, int *status)
{
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    float *buf = reinterpret_cast<float *>(smem_raw);  // 2 stages x 3W rows x 32
    __shared__ __align__(8) uint64_t full[2];
    constexpr uint32_t kBytes = 3 * W * 32 * 4;
    const int lane = threadIdx.x;
    const int64_t n0 = (int64_t)blockIdx.x * 32;
    const int64_t n = n0 + lane;
    const bool act = n < N;
    const int64_t nwin = (M + W - 1) / W;
    auto issue = [&](int s, int64_t w) {
        float *b = buf + (size_t)s * 3 * W * 32;
        mbar_arrive_expect_tx(&full[s], kBytes);
        tma_load_2d(b, &tC, (int)n0, (int)(w * W), &full[s]);
        tma_load_2d(b + W * 32, &tA, (int)n0, (int)(w * W), &full[s]);
        tma_load_2d(b + 2 * W * 32, &tB, (int)n0, (int)(w * W), &full[s]);
    };
    if (lane == 0) {
        for (int s = 0; s < 2; s++) mbar_init(&full[s], 1);
        fence_barrier_init();
    }
    __syncwarp();
    if (lane == 0) {
        issue(0, 0);
        if (nwin > 1) issue(1, 1);
    }
    float l = act ? u0[n] : 0.0f;
    for (int64_t w = 0; w < nwin; w++) {
        const int s = (int)(w & 1);
        if (!mbar_wait(&full[s], (uint32_t)((w >> 1) & 1))) {
            if (status) atomicCAS(status, 0, (int)kStatusTmaWaitTimeout);
            return;
        }
        const float *b = buf + (size_t)s * 3 * W * 32 + lane;
        const int nm = (int)((M - w * W) < W ? (M - w * W) : W);
        for (int j = 0; j < nm; j++) {
            const int64_t m = w * W + j;
            if (act) Lo[m * N + n] = __fsub_rn(l, __fmul_rn(margin, __fadd_rn(fabsf(l), 1.0f)));
            const float c = b[j * 32], a = b[(W + j) * 32], bb = b[(2 * W + j) * 32];
            const float lin = mul_add_rn(a, l, bb);
            l = c < lin ? c : lin;
        }
        __syncwarp();
        if (lane == 0 && w + 2 < nwin) issue(s, w + 2);
    }
}

bool env_carry_staged(const float *u0, const float *EC, const float *EA, const float *EB, float *Lo, int64_t N,
                      int64_t M, float margin, cudaStream_t s)
{
    constexpr int W = 64;
    if (N % 4 || M < 1) return false;
    const void *p[] = {u0, EC, EA, EB, Lo};
    for (const void *q : p)
        if ((uintptr_t)q & 15) return false;
    CUtensorMap t[3];
    if (!make_tmap_2d(&t[0], EC, N, M, 32, W) || !make_tmap_2d(&t[1], EA, N, M, 32, W) ||
        !make_tmap_2d(&t[2], EB, N, M, 32, W))
        return false;
    const size_t smem = (size_t)2 * 3 * W * 32 * 4;
    auto kern = k_env_carry_staged<W>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    count_launches(1);
    kern<<<(unsigned)((N + 31) / 32), 32, smem, s>>>(t[0], t[1], t[2], u0, Lo, N, M, margin, device_status_ptr());
    return true;
}

template <int K, int W>
static bool launch_carry(const float *I, const float *u0, const float *MA, const float *MB, const float *MX,
                         const float *MC, const int32_t *MN, const int32_t *OVF, float *Starts, int64_t N, int64_t M,
                         int64_t L, float beta, float theta, float u_r, cudaStream_t s)
{
    using St = CarryStage<K, W>;
    CUtensorMap t[6];
    if (!make_tmap_2d_typed(&t[0], MA, false, N, M, 32, W) || !make_tmap_2d_typed(&t[1], MB, false, N, M, 32, W) ||
        !make_tmap_2d_typed(&t[2], MN, true, N, M, 32, W) || !make_tmap_2d_typed(&t[3], OVF, true, N, M, 32, W) ||
        !make_tmap_2d_typed(&t[4], MX, false, N, M * K, 32, W * K) ||
        !make_tmap_2d_typed(&t[5], MC, false, N, M * K, 32, W * K))
        return false;
    const size_t smem = (size_t)2 * St::kRows * 32 * 4;
    auto kern = k_carry_staged<K, W>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    count_launches(1);
    kern<<<(unsigned)((N + 31) / 32), 32, smem, s>>>(t[0], t[1], t[2], t[3], t[4], t[5], I, u0, Starts, N, M, L, beta,
                                                      theta, u_r, device_status_ptr());
    return true;
}

bool carry_staged(const float *I, const float *u0, const float *MA, const float *MB, const float *MX, const float *MC,
                  const int32_t *MN, const int32_t *OVF, float *Starts, int64_t N, int64_t M, int64_t L, int K,
                  float beta, float theta, float u_r, cudaStream_t s)
{
    if (N % 4 || M < 1) return false;
    const void *p[] = {MA, MB, MX, MC, MN, OVF, Starts, I, u0};
    for (const void *q : p)
        if ((uintptr_t)q & 15) return false;
    // K is the row stride of the breakpoint slabs: the template K must equal it
    switch (K) {
    case 1: return launch_carry<1, 16>(I, u0, MA, MB, MX, MC, MN, OVF, Starts, N, M, L, beta, theta, u_r, s);
    case 2: return launch_carry<2, 16>(I, u0, MA, MB, MX, MC, MN, OVF, Starts, N, M, L, beta, theta, u_r, s);
    case 4: return launch_carry<4, 16>(I, u0, MA, MB, MX, MC, MN, OVF, Starts, N, M, L, beta, theta, u_r, s);
    case 8: return launch_carry<8, 16>(I, u0, MA, MB, MX, MC, MN, OVF, Starts, N, M, L, beta, theta, u_r, s);
    case 16: return launch_carry<16, 16>(I, u0, MA, MB, MX, MC, MN, OVF, Starts, N, M, L, beta, theta, u_r, s);
    case 32: return launch_carry<32, 8>(I, u0, MA, MB, MX, MC, MN, OVF, Starts, N, M, L, beta, theta, u_r, s);
    case 64: return launch_carry<64, 4>(I, u0, MA, MB, MX, MC, MN, OVF, Starts, N, M, L, beta, theta, u_r, s);
    default: return false;  // other capacities use the plain carry
    }
}

}  // namespace lifb
