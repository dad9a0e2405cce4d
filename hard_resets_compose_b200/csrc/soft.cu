// The soft-reset LIF (subtractive reset u <- v - theta): the model class the
// reference keeps beside the hard reset for its fitting experiments
// (lifscan/triton_lif.py:1035-1082, 1139-1198; lifscan/triton_soft.py).
//
//   lifb_soft_serial_fwd   soft_serial_forward(_tiled): one pass, bit-identical to
//                          the reference's fp32 soft recurrence (the TMA replay
//                          kernel with the reset chosen at compile time)
//   lifb_soft_scan_fwd     soft_scan_forward: exact.  The reference composes
//                          interval maps (Theorem 7 of its paper); here the same
//                          speculative segments as the hard reset (lead-ins,
//                          segment replay, resynchronising fix-up).  A soft reset
//                          forgets its start only as fast as beta^t rounds the
//                          difference away (~1500-3000 rows at beta = 0.99, never
//                          at beta = 1), so wrong guesses cost longer fix-ups;
//                          the result is exact either way.
//   lifb_soft_serial_bwd   soft_serial_backward(_auto): the detached-reset adjoint
//                          lam_t = gs_t sigma'(v_t) + beta lam_{t+1} from U and I
//   lifb_soft_adjoint_v    soft_adjoint_fft: the same recurrence from V; the
//                          reference convolves in float64 by FFT, here it is the
//                          fp32 reverse sweep (within the 1e-5 gradient bar)
//
// The soft reset is the affine reset u <- gamma*v + delta at gamma = 1, delta =
// -theta (fl(1*v) = v, so fl(v + (-theta)) = fl(v - theta) bit for bit): every
// entry point here runs the affine kernels of aff.cu with those constants.
#include <cstdio>

#include "lifb_common.cuh"
#include "lifb_internal.h"

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
}  // namespace

extern "C" {

int lifb_soft_serial_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                         float theta, void *stream)
{
    LIFB_RANGE("lifb_soft_serial_fwd");
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_soft_serial_fwd: negative size");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !U || !S) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_soft_serial_fwd: null pointer");
    lifb::serial_fwd_aff(I, u0, U, S, T, N, beta, theta, 1.0f, -theta, false, (cudaStream_t)stream);
    return done("lifb_soft_serial_fwd");
}

int lifb_soft_scan_fwd(const float *I, const float *u0, float *U, float *S, int64_t T, int64_t N, float beta,
                       float theta, int64_t L, int64_t W, void *workspace, size_t workspace_bytes, void *stream)
{
    LIFB_RANGE("lifb_soft_scan_fwd");
    if (T < 0 || N < 0 || L <= 0 || W < 0 || (T > 0 && T % L))
        return fail(LIFB_ERR_INVALID_ARGUMENT,
                    "lifb_soft_scan_fwd: T must be a multiple of the segment length L > 0, W >= 0");
    if (T / L > 65535) return fail(LIFB_ERR_UNSUPPORTED, "lifb_soft_scan_fwd: more than 65535 segments");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !U || !S) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_soft_scan_fwd: null pointer");
    if (!lifb::aff_scan_fwd(I, u0, U, S, T, N, beta, theta, 1.0f, -theta, L, W, workspace, workspace_bytes,
                            (cudaStream_t)stream))
        return fail(LIFB_ERR_WORKSPACE, "lifb_soft_scan_fwd: workspace missing, misaligned or too small "
                                        "(lifb_scan_fwd_spec_workspace_bytes)");
    return done("lifb_soft_scan_fwd");
}

int lifb_soft_serial_bwd(const float *I, const float *u0, const float *U, const float *GS, float *Lam, int64_t T,
                         int64_t N, float beta, float theta, float alpha, void *stream)
{
    LIFB_RANGE("lifb_soft_serial_bwd");
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_soft_serial_bwd: negative size");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !U || !GS || !Lam) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_soft_serial_bwd: null pointer");
    lifb::serial_bwd_aff(I, u0, U, GS, Lam, T, N, beta, theta, alpha, 1.0f, false, (cudaStream_t)stream);
    return done("lifb_soft_serial_bwd");
}

int lifb_soft_adjoint_v(const float *V, const float *GS, float *Lam, int64_t T, int64_t N, float beta, float theta,
                        float alpha, void *stream)
{
    LIFB_RANGE("lifb_soft_adjoint_v");
    if (T < 0 || N < 0) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_soft_adjoint_v: negative size");
    if (T == 0 || N == 0) return LIFB_OK;
    if (!V || !GS || !Lam) return fail(LIFB_ERR_INVALID_ARGUMENT, "lifb_soft_adjoint_v: null pointer");
    lifb::serial_bwd_aff(V, nullptr, nullptr, GS, Lam, T, N, beta, theta, alpha, 1.0f, true, (cudaStream_t)stream);
    return done("lifb_soft_adjoint_v");
}

}  // extern "C"
