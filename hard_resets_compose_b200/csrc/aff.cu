// The affine-reset LIF (u <- gamma*v + delta on a spike, 0 <= gamma <= 1): the
// family of lifscan/triton_affine.py, which contains the hard reset (gamma = 0,
// delta = u_r) and the soft reset (gamma = 1, delta = -theta).
//
//   lifb_aff_serial_fwd    aff_serial_forward (triton_affine.py:158-162): one pass,
//                          v = fl(fl(beta*u) + x), s = v >= theta,
//                          u' = s ? fl(fl(gamma*v) + delta) : v
//   lifb_aff_scan_fwd      aff_scan_forward (triton_affine.py:165-199), exact.  The
//                          reference builds piecewise-affine chunk maps between a
//                          min-affine and a max-affine envelope; here the
//                          speculative segments of the hard reset (W-row lead-ins
//                          from r(theta) = gamma*theta + delta, all segments replayed
//                          at once, resynchronising fix-up).  A reset maps every
//                          potential >= theta through the same contraction gamma, so
//                          two trajectories merge as fast as beta^t and gamma^spikes
//                          round their difference away.
//   lifb_aff_adjoint       the adjoint of LIFAffineFn.backward (triton_affine.py:
//                          230-238): lam_t = gS_t sigma'(v_t) + a_t lam_{t+1},
//                          a_t = beta*gamma at a spike and beta elsewhere (detached
//                          spike), lam_T = 0.  The reference runs a Hillis-Steele
//                          scan over [T, N] (reverse_affine_scan, :202-211); here
//                          one reverse sweep per neuron through the TMA adjoint
//                          kernel, s recomputed from U and I.
//   lifb_aff_serial_fwd_v  the serial forward writing V (pre-reset potentials)
//                          in place of U: the layer's single-pass forward
//   lifb_aff_adjoint_v     the adjoint from V and u0 with the parameter sums of
//                          LIFAffineFn.backward fused into the same sweep (one
//                          read of V and GS, one write of Lam: 12 B per
//                          neuron-step instead of 16 for the adjoint plus 16
//                          for a separate parameter pass)
//   lifb_reverse_linear_scan  reverse_affine_scan itself for any (a, b) [T, N]:
//                          out_t = a_t out_{t+1} + b_t, out_T = 0, fp32 in order.
#include <cstdio>

#include "lifb_common.cuh"
#include "lifb_internal.h"

namespace lifb {

bool aff_scan_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta, float theta,
                  float gamma, float delta, int64_t L, int64_t W, void *workspace, size_t workspace_bytes,
                  cudaStream_t s)
{
    const int64_t NS = T / L;
    if (NS == 1 || W == 0) {
        serial_fwd_aff(I, u0, U, S, T, N, beta, theta, gamma, delta, false, s);
        return true;
    }
    const size_t one = ((size_t)NS * N * 4 + 255) / 256 * 256;
    if (!workspace || (uintptr_t)workspace % 256 || workspace_bytes < 4 * one) return false;
    char *b = (char *)workspace;
    float *Starts = (float *)b, *Ends = (float *)(b + one), *EndsNew = (float *)(b + 2 * one);
    int32_t *Changed = (int32_t *)(b + 3 * one);
    const Reset rs = affine_reset(gamma, delta);
    // lead-ins start from the value a just-spiking neuron resets to
    const float g_theta = gamma * theta;
    const float r_theta = g_theta + delta;
    // segments led in and replayed in one launch, then the exact fix-up
    if (fwd_replay_tma(I, u0, nullptr, U, S, Ends, T, N, L, beta, theta, r_theta, s, 1, W, Starts, false, rs)) {
        fwd_fixup(I, Starts, 1, U, S, Ends, EndsNew, Changed, N, NS, L, beta, theta, r_theta, nullptr, s, rs);
    } else {
        // the TMA path does not apply: the serial pass (exact, no fix-up needed)
        serial_fwd_aff(I, u0, U, S, T, N, beta, theta, gamma, delta, false, s);
    }
    return true;
}

constexpr int kRevBlock = 128;

// One thread per column, rows in batches of kB loaded ahead of the sweep.
template <int kB>
__global__ void __launch_bounds__(kRevBlock) k_reverse_linear(const float *__restrict__ A, const float *__restrict__ B,
                                                              float *__restrict__ Out, int64_t T, int64_t N)
{
    const int64_t n = (int64_t)blockIdx.x * kRevBlock + threadIdx.x;
    if (n >= N) return;
    float acc = 0.0f;
    for (int64_t tend = T; tend > 0; tend -= kB) {
        const int64_t t0 = tend - kB > 0 ? tend - kB : 0;
        const int cnt = (int)(tend - t0);
        float a[kB], b[kB];
#pragma unroll
        for (int d = 0; d < kB; d++)
            if (d < cnt) {
                a[d] = __ldg(A + (t0 + d) * N + n);
                b[d] = __ldg(B + (t0 + d) * N + n);
            }
#pragma unroll
        for (int d = kB - 1; d >= 0; d--)
            if (d < cnt) {
                acc = __fadd_rn(__fmul_rn(a[d], acc), b[d]);
                Out[(t0 + d) * N + n] = acc;
            }
    }
}

}  // namespace lifb

namespace {
int fail(int st, const char *msg)
{
    lifb::set_last_error(msg);
    return st;
}

int done(const char *who)
{
    if (cudaGetLastError() != cudaSuccess) {
        char msg[128];
        snprintf(msg, sizeof msg, "%s: launch failed", who);
        return fail(LIFB_ERR_CUDA, msg);
    }
    lifb::set_last_error("");
    return LIFB_OK;
}

bool bad_gamma(float gamma) { return !(gamma >= 0.0f && gamma <= 1.0f); }
}  // namespace

extern "C" {

int lifb_aff_serial_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                        float theta, float gamma, float delta, void *stream)
{
    LIFB_RANGE("lifb_aff_serial_fwd");
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_aff_serial_fwd: negative size");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !U || !S) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_aff_serial_fwd: null pointer");
    lifb::serial_fwd_aff(I, u0, U, S, T, N, beta, theta, gamma, delta, false, (cudaStream_t)stream);
    return done("lifb_aff_serial_fwd");
}

int lifb_aff_scan_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                      float theta, float gamma, float delta, int64_t L, int64_t W, void *workspace,
                      size_t workspace_bytes, void *stream)
{
    LIFB_RANGE("lifb_aff_scan_fwd");
    if (T < 0 || N < 0 || L <= 0 || W < 0 || (T > 0 && T % L))
        return fail(LIFB_ERR_INVALID_ARGUMENT,
                    "lifb_aff_scan_fwd: T must be a multiple of the segment length L > 0, W >= 0");
    if (bad_gamma(gamma)) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_aff_scan_fwd: gamma must be in [0, 1]");
    if (T / L > 65535) return fail(LIFB_ERR_UNSUPPORTED, "lifb_aff_scan_fwd: more than 65535 segments");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !U || !S) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_aff_scan_fwd: null pointer");
    if (!lifb::aff_scan_fwd(I, u0, U, S, T, N, beta, theta, gamma, delta, L, W, workspace, workspace_bytes,
                            (cudaStream_t)stream))
        return fail(LIFB_ERR_WORKSPACE, "lifb_aff_scan_fwd: workspace missing, misaligned or too small "
                                        "(lifb_scan_fwd_spec_workspace_bytes)");
    return done("lifb_aff_scan_fwd");
}

int lifb_aff_adjoint(const float *I, const float *u0, const float *U, const float *GS, float *Lam, int64_t T,
                     int64_t N, float beta, float theta, float alpha, float gamma, void *stream)
{
    LIFB_RANGE("lifb_aff_adjoint");
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_aff_adjoint: negative size");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !U || !GS || !Lam) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_aff_adjoint: null pointer");
    lifb::serial_bwd_aff(I, u0, U, GS, Lam, T, N, beta, theta, alpha, gamma, false, (cudaStream_t)stream);
    return done("lifb_aff_adjoint");
}

int lifb_aff_serial_fwd_v(const float *I, const float *u0, float *V, float *S, int64_t T, int64_t N, float beta,
                          float theta, float gamma, float delta, void *stream)
{
    LIFB_RANGE("lifb_aff_serial_fwd_v");
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_aff_serial_fwd_v: negative size");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !V || !S) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_aff_serial_fwd_v: null pointer");
    lifb::serial_fwd_aff(I, u0, V, S, T, N, beta, theta, gamma, delta, true, (cudaStream_t)stream);
    return done("lifb_aff_serial_fwd_v");
}

int lifb_aff_adjoint_v(const float *V, const float *u0, const float *GS, float *Lam, double *param_sums, int64_t T,
                       int64_t N, float beta, float theta, float alpha, float gamma, float delta, void *stream)
{
    LIFB_RANGE("lifb_aff_adjoint_v");
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_aff_adjoint_v: negative size");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!V || !GS || !Lam || (param_sums && !u0))
        return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_aff_adjoint_v: null pointer (param_sums needs u0)");
    lifb::serial_bwd_aff(V, u0, nullptr, GS, Lam, T, N, beta, theta, alpha, gamma, true, (cudaStream_t)stream, delta,
                         param_sums);
    return done("lifb_aff_adjoint_v");
}

int lifb_reverse_linear_scan(const float *A, const float *B, float *Out, int64_t T, int64_t N, void *stream)
{
    LIFB_RANGE("lifb_reverse_linear_scan");
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_reverse_linear_scan: negative size");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!A || !B || !Out) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_reverse_linear_scan: null pointer");
    lifb::count_launches(1);
    const unsigned g = (unsigned)((N + lifb::kRevBlock - 1) / lifb::kRevBlock);
    lifb::k_reverse_linear<8><<<g, lifb::kRevBlock, 0, (cudaStream_t)stream>>>(A, B, Out, T, N);
    return done("lifb_reverse_linear_scan");
}

}  // extern "C"
