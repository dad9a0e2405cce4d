// Tiled affine-scan backward with the surrogate fused in
// (lifscan/triton_lif.py:512-526 scan_backward_tiled):
//   k_bwd_chunk   chunk adjoint map lam_start = P*lam_end + Q   bwd_chunk_tiled_kernel :421-457
//   k_bwd_carry   reverse carry over chunks -> LamEnd[m]        bwd_carry_kernel       :197-208
//   k_bwd_replay  chunk replay from LamEnd -> Lam               bwd_tiled_kernel       :382-418
// The coefficients (a_t, b_t) come from lif_coef (triton_lif.py:42-50) with v
// recomputed from U[t-1] (u0 at t = 0) and I.
#include "lifb_common.cuh"
#include "lifb_internal.h"

namespace lifb {

constexpr int kBwBlock = 128;

__device__ __forceinline__ void coef_at(const float *__restrict__ I, const float *__restrict__ u0,
                                        const float *__restrict__ U, const float *__restrict__ S,
                                        const float *__restrict__ GS, const float *__restrict__ GU, int64_t t,
                                        int64_t N, int64_t n, float beta, float theta, float u_r, float alpha,
                                        bool detach, float &a, float &b)
{
    int64_t o = t * N + n;
    float up = t > 0 ? __ldg(U + o - N) : __ldg(u0 + n);
    float gu = GU ? __ldg(GU + o) : 0.0f;
    float sv = S ? __ldg(S + o) : -1.0f;  // -1: recompute from v
    lif_coef(up, sv, __ldg(I + o), __ldg(GS + o), gu, beta, theta, u_r, alpha, detach, a, b);
}

__global__ void __launch_bounds__(kBwBlock) k_bwd_chunk(const float *__restrict__ I, const float *__restrict__ u0,
                                                        const float *__restrict__ U, const float *__restrict__ S,
                                                        const float *__restrict__ GS, const float *__restrict__ GU,
                                                        float *__restrict__ P, float *__restrict__ Q, int64_t N,
                                                        int C, float beta, float theta, float u_r, float alpha,
                                                        bool detach)
{
    int64_t n = (int64_t)blockIdx.x * kBwBlock + threadIdx.x;
    if (n >= N) return;
    int64_t m = blockIdx.y;
    float p = 1.0f, q = 0.0f;
#pragma unroll 4
    for (int i = 0; i < C; i++) {
        int64_t t = m * C + C - 1 - i;
        float a, b;
        coef_at(I, u0, U, S, GS, GU, t, N, n, beta, theta, u_r, alpha, detach, a, b);
        q = b + a * q;
        p = a * p;
    }
    P[m * N + n] = p;
    Q[m * N + n] = q;
}

__global__ void __launch_bounds__(kBwBlock) k_bwd_carry(const float *__restrict__ P, const float *__restrict__ Q,
                                                        float *__restrict__ LamEnd, int64_t N, int64_t M)
{
    int64_t n = (int64_t)blockIdx.x * kBwBlock + threadIdx.x;
    if (n >= N) return;
    float lam = 0.0f;
#pragma unroll 4
    for (int64_t i = 0; i < M; i++) {
        int64_t m = M - 1 - i;
        LamEnd[m * N + n] = lam;
        lam = Q[m * N + n] + P[m * N + n] * lam;
    }
}

__global__ void __launch_bounds__(kBwBlock) k_bwd_replay(const float *__restrict__ I, const float *__restrict__ u0,
                                                         const float *__restrict__ U, const float *__restrict__ S,
                                                         const float *__restrict__ GS, const float *__restrict__ GU,
                                                         const float *__restrict__ LamEnd, float *__restrict__ Lam,
                                                         int64_t N, int C, float beta, float theta, float u_r,
                                                         float alpha, bool detach)
{
    int64_t n = (int64_t)blockIdx.x * kBwBlock + threadIdx.x;
    if (n >= N) return;
    int64_t m = blockIdx.y;
    float lam = LamEnd[m * N + n];
#pragma unroll 4
    for (int i = 0; i < C; i++) {
        int64_t t = m * C + C - 1 - i;
        float a, b;
        coef_at(I, u0, U, S, GS, GU, t, N, n, beta, theta, u_r, alpha, detach, a, b);
        lam = b + a * lam;
        Lam[t * N + n] = lam;
    }
}

void grid_scan_bwd(const float *I, const float *u0, const float *U, const float *S, const float *GS,
                   const float *GU, float *Lam, BwdScratch &w, int64_t T, int64_t N, int C, float beta,
                   float theta, float u_r, float alpha, bool detach, cudaStream_t s)
{
    int64_t M = T / C;
    unsigned nb = (unsigned)((N + kBwBlock - 1) / kBwBlock);
    if (!bwd_tma(1, I, u0, U, S, GS, GU, nullptr, nullptr, w.P, w.Q, T, N, C, beta, theta, u_r, alpha, detach, s)) {
        count_launches(1);
        k_bwd_chunk<<<dim3(nb, (unsigned)M), kBwBlock, 0, s>>>(I, u0, U, S, GS, GU, w.P, w.Q, N, C, beta, theta,
                                                                u_r, alpha, detach);
    }
    count_launches(1);
    k_bwd_carry<<<nb, kBwBlock, 0, s>>>(w.P, w.Q, w.LamEnd, N, M);
    if (!bwd_tma(0, I, u0, U, S, GS, GU, w.LamEnd, Lam, nullptr, nullptr, T, N, C, beta, theta, u_r, alpha, detach,
                 s)) {
        count_launches(1);
        k_bwd_replay<<<dim3(nb, (unsigned)M), kBwBlock, 0, s>>>(I, u0, U, S, GS, GU, w.LamEnd, Lam, N, C, beta,
                                                                 theta, u_r, alpha, detach);
    }
}

}  // namespace lifb
