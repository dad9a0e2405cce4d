// Parameter gradients of the hard-reset LIF (the fitting layer of
// lifscan/fit.py:15-61), read off the adjoint lam_t = dL/dv_t in one pass:
//   dL/dbeta  = sum_t lam_t u_{t-1}
//   dL/dtheta = -sum_t gS_t sigma'(v_t - theta)      (detached reset)
//   dL/du_r   = sum_t s_t beta lam_{t+1}             (lam_T = 0)
// with v_t = fl(fl(beta u_{t-1}) + x_t), s_t = [v_t >= theta] recomputed bit for
// bit, sigma' = alpha sig (1 - sig).  The reference forms u_{t-1}, v_t, the
// surrogate and three products as [T, N] tensors (fit.py:36-47); here every
// (chunk of rows, neuron) thread reads I, U, GS and Lam once (16 B per
// neuron-step) and accumulates in fp64; the caller sums the [3, M, N] partials.
//
// The affine reset u = s ? gamma v + delta : v (LIFAffineFn.backward,
// lifscan/triton_affine.py:230-238) adds one row: with dL/du_t = beta lam_{t+1},
//   dL/ddelta = sum_t s_t beta lam_{t+1}   (the du_r row above)
//   dL/dgamma = sum_t s_t v_t beta lam_{t+1}
// and dL/dbeta = sum_t lam_t u_{t-1} as before (U holds the post-reset u).
#include <cstdio>

#include "lifb_common.cuh"
#include "lifb_internal.h"
#include "tma.cuh"

namespace lifb {

constexpr int kPgBlock = 128;

template <bool AFF>
__global__ void __launch_bounds__(kPgBlock) k_param_partials(const float *__restrict__ I, const float *__restrict__ u0,
                                                             const float *__restrict__ U, const float *__restrict__ GS,
                                                             const float *__restrict__ Lam, double *__restrict__ part,
                                                             int64_t T, int64_t N, int64_t C, float beta, float theta,
                                                             float alpha)
{
    const int64_t n = (int64_t)blockIdx.x * kPgBlock + threadIdx.x;
    const int64_t m = blockIdx.y, M = gridDim.y;
    if (n >= N) return;
    const int64_t t0 = m * C, t1 = (t0 + C < T) ? t0 + C : T;
    const float k2 = alpha * 1.4426950408889634f;  // exp(x) = 2^(x log2 e)
    double db = 0.0, dt = 0.0, dr = 0.0, dg = 0.0;
    constexpr int kB = 8;
    for (int64_t b = t0; b < t1; b += kB) {
        float up[kB], x[kB], gs[kB], lm[kB], ln[kB];
#pragma unroll
        for (int q = 0; q < kB; q++) {
            const int64_t t = b + q;
            if (t < t1) {
                up[q] = t > 0 ? U[(t - 1) * N + n] : u0[n];
                x[q] = I[t * N + n];
                gs[q] = GS[t * N + n];
                lm[q] = Lam[t * N + n];
                ln[q] = t + 1 < T ? Lam[(t + 1) * N + n] : 0.0f;
            }
        }
#pragma unroll
        for (int q = 0; q < kB; q++) {
            if (b + q < t1) {
                const float v = __fadd_rn(__fmul_rn(beta, up[q]), x[q]);
                const float e = ex2_approx(k2 * (theta - v));
                const float sig = rcp_approx(1.0f + e);
                const float sg = alpha * sig * (1.0f - sig);
                db += (double)lm[q] * (double)up[q];
                dt -= (double)gs[q] * (double)sg;
                if (v >= theta) {
                    const double bl = (double)beta * (double)ln[q];
                    dr += bl;
                    if (AFF) dg += (double)v * bl;
                }
            }
        }
    }
    part[(0 * M + m) * N + n] = db;
    part[(1 * M + m) * N + n] = dt;
    part[(2 * M + m) * N + n] = dr;
    if (AFF) part[(3 * M + m) * N + n] = dg;
}

}  // namespace lifb

extern "C" {

int lifb_param_grad_chunks(int64_t T, int64_t N)
{
    LIFB_RANGE("lifb_param_grad_chunks");
    if (T <= 0 || N <= 0) return 0;
    // enough (chunk, neuron) threads for ~8 warps per SM, chunks of >= 64 rows
    const int64_t want = (8 * 148 * 32 + N - 1) / N;
    int64_t M = want < 1 ? 1 : want;
    const int64_t max_m = (T + 63) / 64;
    if (M > max_m) M = max_m;
    if (M > 65535) M = 65535;
    return (int)M;
}

static int param_partials(const char *who, bool aff, const float *I, const float *u0, const float *U,
                          const float *GS, const float *Lam, double *partials, int64_t T, int64_t N, float beta,
                          float theta, float alpha, int M, void *stream)
{
    char msg[160];
    if (T < 0 || N < 0 || M <= 0 || M > 65535) {
        snprintf(msg, sizeof msg, "%s: bad sizes (need T, N >= 0 and 1 <= M <= 65535)", who);
        lifb::set_last_error(msg);
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !U || !GS || !Lam || !partials) {
        snprintf(msg, sizeof msg, "%s: null pointer", who);
        lifb::set_last_error(msg);
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    const int64_t C = (T + M - 1) / M;  // chunks past row T-1 write zeros
    lifb::count_launches(1);
    dim3 g((unsigned)((N + lifb::kPgBlock - 1) / lifb::kPgBlock), (unsigned)M);
    cudaStream_t s = (cudaStream_t)stream;
    if (aff)
        lifb::k_param_partials<true><<<g, lifb::kPgBlock, 0, s>>>(I, u0, U, GS, Lam, partials, T, N, C, beta, theta,
                                                                  alpha);
    else
        lifb::k_param_partials<false><<<g, lifb::kPgBlock, 0, s>>>(I, u0, U, GS, Lam, partials, T, N, C, beta, theta,
                                                                   alpha);
    if (cudaGetLastError() != cudaSuccess) {
        snprintf(msg, sizeof msg, "%s: launch failed", who);
        lifb::set_last_error(msg);
        return LIFB_ERR_CUDA;
    }
    lifb::set_last_error("");
    return LIFB_OK;
}

int lifb_param_grad_partials(const float *I, const float *u0, const float *U, const float *GS, const float *Lam,
                             double *partials, int64_t T, int64_t N, float beta, float theta, float alpha, int M,
                             void *stream)
{
    LIFB_RANGE("lifb_param_grad_partials");
    return param_partials("lifb_param_grad_partials", false, I, u0, U, GS, Lam, partials, T, N, beta, theta, alpha,
                          M, stream);
}

int lifb_aff_param_grad_partials(const float *I, const float *u0, const float *U, const float *GS, const float *Lam,
                                 double *partials, int64_t T, int64_t N, float beta, float theta, float alpha, int M,
                                 void *stream)
{
    LIFB_RANGE("lifb_aff_param_grad_partials");
    return param_partials("lifb_aff_param_grad_partials", true, I, u0, U, GS, Lam, partials, T, N, beta, theta,
                          alpha, M, stream);
}

}  // extern "C"
