// lif_tuned's layer with the pre-reset potential saved instead of the state.
//
// The reference's layer saves U (and S) for its backward (lifscan/triton_lif.py:
// 654-683), which then recomputes v_t = fl(fl(beta*u_{t-1}) + x_t) from U and I.
// v_t alone determines everything the detached-reset adjoint needs: the spike
// s_t = [v_t >= theta], the surrogate at v_t, and so a_t, c_t.  Saving V in
// place of U (same bytes written) lets the adjoint read V and GS only:
// forward 12 + adjoint 12 = 24 bytes per neuron-step instead of 12 + 16.
// S, dI and du0 are those of the reference's layer (S bit for bit).
#include <cstdio>

#include "lifb_common.cuh"
#include "lifb_internal.h"

namespace {
constexpr size_t kAl = 256;
size_t al(size_t x) { return (x + kAl - 1) / kAl * kAl; }

int done(const char *who)
{
    if (cudaGetLastError() != cudaSuccess) {
        char msg[128];
        snprintf(msg, sizeof msg, "%s: launch failed", who);
        lifb::set_last_error(msg);
        return LIFB_ERR_CUDA;
    }
    lifb::set_last_error("");
    return LIFB_OK;
}
}  // namespace

extern "C" {

int lifb_serial_fwd_v(const float *I, const float *u0, float *V, float *S, int64_t T, int64_t N, float beta,
                      float theta, float u_r, void *stream)
{
    LIFB_RANGE("lifb_serial_fwd_v");
    if (T < 0 || N < 0) {
        lifb::set_last_error("lifb_serial_fwd_v: negative size");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (T == 0 || N == 0) return LIFB_OK;
    if (!I || !u0 || !V || !S) {
        lifb::set_last_error("lifb_serial_fwd_v: null pointer");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    lifb::serial_fwd_v(I, u0, V, S, T, N, beta, theta, u_r, (cudaStream_t)stream);
    return done("lifb_serial_fwd_v");
}

size_t lifb_lif_bwd_v_workspace_bytes(int64_t T, int64_t N, int C)
{
    if (T <= 0 || N <= 0 || C <= 0 || T % C) return 0;
    return 3 * al((size_t)(T / C) * N * 4);
}

int lifb_lif_bwd_v(const float *V, const float *GS, float *Lam, int64_t T, int64_t N, float beta, float theta,
                   float alpha, int C, void *workspace, size_t workspace_bytes, void *stream)
{
    LIFB_RANGE("lifb_lif_bwd_v");
    if (T < 0 || N < 0 || C <= 0 || (T > 0 && T % C)) {
        lifb::set_last_error("lifb_lif_bwd_v: T must be a multiple of the chunk length C > 0");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    if (T == 0 || N == 0) return LIFB_OK;
    if (!V || !GS || !Lam) {
        lifb::set_last_error("lifb_lif_bwd_v: null pointer");
        return LIFB_ERR_INVALID_ARGUMENT;
    }
    cudaStream_t s = (cudaStream_t)stream;
    const int64_t M = T / C;
    if (M == 1) {
        lifb::serial_bwd_v(V, GS, Lam, T, N, beta, theta, alpha, s);
        return done("lifb_lif_bwd_v");
    }
    if (M > 65535) {
        lifb::set_last_error("lifb_lif_bwd_v: more than 65535 chunks");
        return LIFB_ERR_UNSUPPORTED;
    }
    if (!workspace || (uintptr_t)workspace % kAl || workspace_bytes < lifb_lif_bwd_v_workspace_bytes(T, N, C)) {
        lifb::set_last_error("lifb_lif_bwd_v: workspace missing, misaligned or too small");
        return LIFB_ERR_WORKSPACE;
    }
    const size_t one = al((size_t)M * N * 4);
    float *P = (float *)workspace, *Q = (float *)((char *)workspace + one);
    int32_t *D = (int32_t *)((char *)workspace + 2 * one);
    // chunks replayed from lam = 0 at once, then the rows above each chunk's
    // last spike corrected by lam_end * beta^k (the D path reads only P, Q, D)
    if (lifb::bwd_tma_v(V, GS, Lam, P, Q, D, T, N, C, beta, theta, alpha, s)) {
        lifb::bwd_fixup(nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, P, Q, D, Lam, N, M, C, beta, theta,
                        alpha, s);
    } else {
        lifb::serial_bwd_v(V, GS, Lam, T, N, beta, theta, alpha, s);
    }
    return done("lifb_lif_bwd_v");
}

}  // extern "C"
