// Serial forward and adjoint: one recurrence per thread, neurons along the
// lanes (coalesced rows of [T, N]), time tiles of D rows prefetched into
// registers one tile ahead.
//   k_serial_fwd  follows fwd_tiled_kernel with M = 1 (lifscan/triton_lif.py:353-379,
//                 serial_forward_tiled :460-466) and fast.serial_forward_nograd
//                 (lifscan/fast.py:69-81) bit for bit.
//   k_serial_bwd  follows bwd_tiled_pf_kernel (lifscan/triton_lif.py:1087-1127)
//                 and fast.serial_backward (lifscan/fast.py:227-239).
#include "lifb_common.cuh"
#include "lifb_internal.h"

namespace lifb {

constexpr int kSerBlock = 128;
constexpr int kSerD = 16;

// VOUT: U receives the pre-reset potential v_t instead of u_t.  AFF: the
// affine reset u = fl(fl(gamma*v) + delta) (gamma = 1, delta = -theta: the
// soft reset).
template <int D, bool VOUT, bool AFF = false>
__global__ void __launch_bounds__(kSerBlock) k_serial_fwd(const float *__restrict__ I, const float *__restrict__ u0,
                                                          float *__restrict__ U, float *__restrict__ S, int64_t T,
                                                          int64_t N, float beta, float theta, float u_r,
                                                          float gamma = 0.0f, float delta = 0.0f)
{
    int64_t n = (int64_t)blockIdx.x * kSerBlock + threadIdx.x;
    if (n >= N) return;
    float u = u0[n];
    const float *p = I + n;
    int64_t Tf = (T / D) * D;
    float cur[D], nxt[D];
    if (Tf > 0) {
#pragma unroll
        for (int d = 0; d < D; d++) cur[d] = __ldg(p + (int64_t)d * N);
    }
    for (int64_t t0 = 0; t0 < Tf; t0 += D) {
        bool more = t0 + D < Tf;
        if (more) {
#pragma unroll
            for (int d = 0; d < D; d++) nxt[d] = __ldg(p + (t0 + D + d) * N);
        }
#pragma unroll
        for (int d = 0; d < D; d++) {
            const float v = __fadd_rn(__fmul_rn(beta, u), cur[d]);
            const bool s = v >= theta;
            u = s ? (AFF ? __fadd_rn(__fmul_rn(gamma, v), delta) : u_r) : v;
            int64_t o = (t0 + d) * N + n;
            U[o] = VOUT ? v : u;
            S[o] = s ? 1.0f : 0.0f;
        }
        if (more) {
#pragma unroll
            for (int d = 0; d < D; d++) cur[d] = nxt[d];
        }
    }
    for (int64_t t = Tf; t < T; t++) {
        const float v = __fadd_rn(__fmul_rn(beta, u), __ldg(p + t * N));
        const bool s = v >= theta;
        u = s ? (AFF ? __fadd_rn(__fmul_rn(gamma, v), delta) : u_r) : v;
        U[t * N + n] = VOUT ? v : u;
        S[t * N + n] = s ? 1.0f : 0.0f;
    }
}

// Reverse sweep from V (pre-reset potentials) and GS: detached reset, s = [v >= theta], no GU.
template <int D>
__global__ void __launch_bounds__(kSerBlock) k_serial_bwd_v(const float *__restrict__ V, const float *__restrict__ GS,
                                                            float *__restrict__ Lam, int64_t T, int64_t N, float beta,
                                                            float theta, float alpha)
{
    int64_t n = (int64_t)blockIdx.x * kSerBlock + threadIdx.x;
    if (n >= N) return;
    float lam = 0.0f;
    for (int64_t tend = T; tend > 0; tend -= D) {
        int64_t t0 = tend - D > 0 ? tend - D : 0;
        int cnt = (int)(tend - t0);
        float v[D], gs[D];
#pragma unroll
        for (int d = 0; d < D; d++) {
            if (d < cnt) {
                const int64_t o = (t0 + d) * N + n;
                v[d] = __ldg(V + o);
                gs[d] = __ldg(GS + o);
            }
        }
#pragma unroll
        for (int dd = D - 1; dd >= 0; dd--) {
            if (dd < cnt) {
                const float s = v[dd] >= theta ? 1.0f : 0.0f;
                const float sig = __frcp_rn(1.0f + __expf(-alpha * (v[dd] - theta)));
                const float sg = alpha * sig * (1.0f - sig);
                lam = gs[dd] * sg + beta * (1.0f - s) * lam;
                Lam[(t0 + dd) * N + n] = lam;
            }
        }
    }
}

// Reverse sweep in tiles of D rows [t0, t0 + cnt), last tile first.
template <int D>
__global__ void __launch_bounds__(kSerBlock) k_serial_bwd(const float *__restrict__ I, const float *__restrict__ u0,
                                                          const float *__restrict__ U, const float *__restrict__ S,
                                                          const float *__restrict__ GS, const float *__restrict__ GU,
                                                          float *__restrict__ Lam, int64_t T, int64_t N, float beta,
                                                          float theta, float u_r, float alpha, bool detach)
{
    int64_t n = (int64_t)blockIdx.x * kSerBlock + threadIdx.x;
    if (n >= N) return;
    float lam = 0.0f;
    float un0 = u0[n];
    for (int64_t tend = T; tend > 0; tend -= D) {
        int64_t t0 = tend - D > 0 ? tend - D : 0;
        int cnt = (int)(tend - t0);
        float x[D], s[D], up[D], gs[D], gu[D];
#pragma unroll
        for (int d = 0; d < D; d++) {
            if (d < cnt) {
                int64_t t = t0 + d;
                int64_t o = t * N + n;
                x[d] = __ldg(I + o);
                s[d] = S ? __ldg(S + o) : -1.0f;
                gs[d] = __ldg(GS + o);
                gu[d] = GU ? __ldg(GU + o) : 0.0f;
                up[d] = t > 0 ? __ldg(U + o - N) : un0;
            }
        }
#pragma unroll
        for (int dd = D - 1; dd >= 0; dd--) {
            if (dd < cnt) {
                float a, b;
                lif_coef(up[dd], s[dd], x[dd], gs[dd], gu[dd], beta, theta, u_r, alpha, detach, a, b);
                lam = b + a * lam;
                Lam[(t0 + dd) * N + n] = lam;
            }
        }
    }
}

void serial_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                float theta, float u_r, cudaStream_t s)
{
    if (fwd_replay_tma(I, u0, nullptr, U, S, nullptr, T, N, T, beta, theta, u_r, s)) return;
    unsigned g = (unsigned)((N + kSerBlock - 1) / kSerBlock);
    count_launches(1);
    k_serial_fwd<kSerD, false><<<g, kSerBlock, 0, s>>>(I, u0, U, S, T, N, beta, theta, u_r);
}

// Affine-reset adjoint (detached reset), one thread per neuron: lam_t =
// gs_t sigma'(v_t) + a_t lam_{t+1}, a_t = beta*gamma at a spike and beta
// elsewhere, with v_t from V (from_v) or from U[t-1] and I[t] (u0 for row 0).
// PGout (optional, [3][N] fp64): the parameter sums (dbeta, dgamma, ddelta) =
// (sum lam_{t+1} u_t + lam_0 u0, sum s_t v_t beta lam_{t+1}, sum s_t beta lam_{t+1})
// with u_t = s_t ? fl(fl(gamma v_t) + delta) : v_t; then u0 must be given.
template <int D>
__global__ void __launch_bounds__(kSerBlock) k_serial_bwd_aff(const float *__restrict__ IV,
                                                              const float *__restrict__ u0,
                                                              const float *__restrict__ U,
                                                              const float *__restrict__ GS, float *__restrict__ Lam,
                                                              int64_t T, int64_t N, float beta, float theta,
                                                              float alpha, float gamma, bool from_v, float delta,
                                                              double *__restrict__ PGout)
{
    int64_t n = (int64_t)blockIdx.x * kSerBlock + threadIdx.x;
    if (n >= N) return;
    float lam = 0.0f;
    const float un0 = from_v ? 0.0f : u0[n];
    const float bg = beta * gamma;
    double pb = 0.0, pgm = 0.0, pdl = 0.0;
    for (int64_t tend = T; tend > 0; tend -= D) {
        int64_t t0 = tend - D > 0 ? tend - D : 0;
        int cnt = (int)(tend - t0);
        float v[D], gs[D];
#pragma unroll
        for (int d = 0; d < D; d++) {
            if (d < cnt) {
                const int64_t t = t0 + d, o = t * N + n;
                const float xv = __ldg(IV + o);
                v[d] = from_v ? xv : __fadd_rn(__fmul_rn(beta, t > 0 ? __ldg(U + o - N) : un0), xv);
                gs[d] = __ldg(GS + o);
            }
        }
#pragma unroll
        for (int dd = D - 1; dd >= 0; dd--) {
            if (dd < cnt) {
                const float sig = __frcp_rn(1.0f + __expf(-alpha * (v[dd] - theta)));
                const bool spk = v[dd] >= theta;
                if (PGout) {  // lam is lam_{t+1} here
                    const float u = spk ? __fadd_rn(__fmul_rn(gamma, v[dd]), delta) : v[dd];
                    pb = fma((double)lam, (double)u, pb);
                    if (spk) {
                        const double bl = (double)beta * (double)lam;
                        pdl += bl;
                        pgm = fma((double)v[dd], bl, pgm);
                    }
                }
                lam = gs[dd] * (alpha * sig * (1.0f - sig)) + (spk ? bg : beta) * lam;
                Lam[(t0 + dd) * N + n] = lam;
            }
        }
    }
    if (PGout) {
        pb = fma((double)lam, (double)u0[n], pb);
        PGout[n] = pb;
        PGout[N + n] = pgm;
        PGout[2 * N + n] = pdl;
    }
}

void serial_fwd_aff(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                    float theta, float gamma, float delta, bool vout, cudaStream_t s)
{
    if (fwd_replay_tma(I, u0, nullptr, U, S, nullptr, T, N, T, beta, theta, 0.0f, s, 1, 0, nullptr, vout,
                       affine_reset(gamma, delta)))
        return;
    unsigned g = (unsigned)((N + kSerBlock - 1) / kSerBlock);
    count_launches(1);
    if (vout)
        k_serial_fwd<kSerD, true, true><<<g, kSerBlock, 0, s>>>(I, u0, U, S, T, N, beta, theta, 0.0f, gamma, delta);
    else
        k_serial_fwd<kSerD, false, true><<<g, kSerBlock, 0, s>>>(I, u0, U, S, T, N, beta, theta, 0.0f, gamma, delta);
}

void serial_bwd_aff(const float *IV, const float *u0, const float *U, const float *GS, float *Lam, int64_t T,
                    int64_t N, float beta, float theta, float alpha, float gamma, bool from_v, cudaStream_t s,
                    float delta, double *PGout)
{
    if (PGout && from_v) {
        if (bwd_tma_aff_pg(IV, u0, GS, Lam, PGout, T, N, beta, theta, alpha, gamma, delta, s)) return;
    } else if (!PGout && bwd_tma_aff(IV, u0, U, GS, Lam, T, N, beta, theta, alpha, gamma, from_v, s)) {
        return;
    }
    unsigned g = (unsigned)((N + kSerBlock - 1) / kSerBlock);
    count_launches(1);
    k_serial_bwd_aff<8><<<g, kSerBlock, 0, s>>>(IV, u0, U, GS, Lam, T, N, beta, theta, alpha, gamma, from_v, delta,
                                                PGout);
}

void serial_fwd_v(const float *I, const float *u0, float *V, float *S, int64_t T, int64_t N, float beta,
                  float theta, float u_r, cudaStream_t s)
{
    if (fwd_replay_tma(I, u0, nullptr, V, S, nullptr, T, N, T, beta, theta, u_r, s, 1, 0, nullptr, true)) return;
    unsigned g = (unsigned)((N + kSerBlock - 1) / kSerBlock);
    count_launches(1);
    k_serial_fwd<kSerD, true><<<g, kSerBlock, 0, s>>>(I, u0, V, S, T, N, beta, theta, u_r);
}

void serial_bwd_v(const float *V, const float *GS, float *Lam, int64_t T, int64_t N, float beta, float theta,
                  float alpha, cudaStream_t s)
{
    if (bwd_tma_v(V, GS, Lam, nullptr, nullptr, nullptr, T, N, T, beta, theta, alpha, s)) return;
    unsigned g = (unsigned)((N + kSerBlock - 1) / kSerBlock);
    count_launches(1);
    k_serial_bwd_v<8><<<g, kSerBlock, 0, s>>>(V, GS, Lam, T, N, beta, theta, alpha);
}

void serial_bwd(const float *I, const float *u0, const float *U, const float *S, const float *GS,
                const float *GU, float *Lam, int64_t T, int64_t N, float beta, float theta, float u_r,
                float alpha, bool detach, cudaStream_t s)
{
    if (bwd_tma(0, I, u0, U, S, GS, GU, nullptr, Lam, nullptr, nullptr, T, N, T, beta, theta, u_r, alpha, detach, s))
        return;
    unsigned g = (unsigned)((N + kSerBlock - 1) / kSerBlock);
    count_launches(1);
    k_serial_bwd<8><<<g, kSerBlock, 0, s>>>(I, u0, U, S, GS, GU, Lam, T, N, beta, theta, u_r, alpha, detach);
}

}  // namespace lifb
