// Shared device helpers of the B200 hard-reset LIF scan.
//
// The per-step arithmetic is the bit-exactness anchor: every kernel that
// produces U or S (serial, replay, repair, carry fallback, map constants) calls
// lif_step(), which rounds beta*u and the sum separately (no FMA), exactly as
// the reference's fp32 serial recurrence (lifscan/fast.py:69-81) and its
// Triton `_step` (lifscan/triton_lif.py:20-25) under the interpreter do.
// Map and envelope arithmetic (lifscan/triton_lif.py:698-779, 828-899) is
// rounded the same way so the maps equal the CPU oracle's bit for bit.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#define LIFB_DEV __device__ __forceinline__

namespace lifb {

constexpr float kInf = __builtin_huge_valf();

// One LIF step: v = fl(fl(beta*u) + x); s = v >= theta; u' = s ? u_r : v.
LIFB_DEV float lif_step(float u, float x, float beta, float theta, float u_r, bool &s)
{
    float v = __fadd_rn(__fmul_rn(beta, u), x);
    s = v >= theta;
    return s ? u_r : v;
}

LIFB_DEV float lif_step_u(float u, float x, float beta, float theta, float u_r)
{
    float v = __fadd_rn(__fmul_rn(beta, u), x);
    return v >= theta ? u_r : v;
}

// The same step with the reset chosen at compile time: the hard reset above,
// or the affine reset u' = s ? fl(fl(gamma*v) + delta) : v of the affine-reset
// model (lifscan/triton_affine.py:20-24 _aff_step).  It contains the soft
// (subtractive) reset (lifscan/triton_lif.py:1037-1049): gamma = 1, delta =
// -theta gives fl(v - theta) bit for bit.
template <bool AFF>
LIFB_DEV float step_r(float u, float x, float beta, float theta, float u_r, float gamma, float delta, bool &s)
{
    const float v = __fadd_rn(__fmul_rn(beta, u), x);
    s = v >= theta;
    return s ? (AFF ? __fadd_rn(__fmul_rn(gamma, v), delta) : u_r) : v;
}

template <bool AFF>
LIFB_DEV float step_r_u(float u, float x, float beta, float theta, float u_r, float gamma, float delta)
{
    bool s;
    return step_r<AFF>(u, x, beta, theta, u_r, gamma, delta, s);
}

// Runtime choice (host-chosen flag, uniform across the grid): the fix-up and
// lead-in kernels, whose cost is not the step.
LIFB_DEV float step_any(float u, float x, float beta, float theta, float u_r, bool aff, float gamma, float delta,
                        bool &s)
{
    const float v = __fadd_rn(__fmul_rn(beta, u), x);
    s = v >= theta;
    return s ? (aff ? __fadd_rn(__fmul_rn(gamma, v), delta) : u_r) : v;
}

// fl(fl(a*b) + c), never contracted to an FMA.
LIFB_DEV float mul_add_rn(float a, float b, float c) { return __fadd_rn(__fmul_rn(a, b), c); }

// Adjoint coefficients of one step (lifscan/triton_lif.py:42-50 `_coef`):
// lam_t = a * lam_{t+1} + b with a = beta*J, b = gs*sigma' + J*gu,
// sigma' = alpha*sig*(1-sig), sig = 1/(1+exp(-alpha*(v-theta))), J = 1-s
// (+ (u_r - v)*sigma' when the reset is not detached).  v is recomputed from
// the saved previous state with the forward's exact rounding.
// s < 0 means "not stored": s = [v >= theta] is recomputed from v, which is
// bit-identical to the forward's spike.
LIFB_DEV void lif_coef(float up, float s, float x, float gs, float gu, float beta, float theta,
                       float u_r, float alpha, bool detach, float &a, float &b)
{
    float v = __fadd_rn(__fmul_rn(beta, up), x);
    if (s < 0.0f) s = v >= theta ? 1.0f : 0.0f;
    float e = __expf(-alpha * (v - theta));
    float sig = __frcp_rn(1.0f + e);
    float sg = alpha * sig * (1.0f - sig);
    float J = 1.0f - s;
    if (detach == false) J = J + (u_r - v) * sg;
    a = beta * J;
    b = gs * sg + J * gu;
}

// Surrogate derivative only (detached reset, gu == 0): b = gs*sigma'(v).
LIFB_DEV float lif_sg(float up, float x, float beta, float theta, float alpha)
{
    float v = __fadd_rn(__fmul_rn(beta, up), x);
    float e = __expf(-alpha * (v - theta));
    float sig = __frcp_rn(1.0f + e);
    return alpha * sig * (1.0f - sig);
}

}  // namespace lifb
