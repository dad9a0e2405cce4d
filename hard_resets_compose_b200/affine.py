"""Drop-in mirror of the reference's `lifscan.triton_affine` (LIF with an
affine reset u <- gamma*v + delta, 0 <= gamma <= 1) on B200 kernels.

    from hard_resets_compose_b200 import affine as A   # was: from lifscan import triton_affine as A
    U, S = A.aff_scan_forward(I, 0.97, 1.0, 0.3, -0.1, u0, C=128, K=32)
    S = A.lif_affine(I, u0, beta, gamma, delta)         # grads for I, u0, beta, gamma, delta

Same names, arguments and return values as lifscan/triton_affine.py.  The
family contains the hard reset (gamma = 0, delta = u_r) and the soft reset
(gamma = 1, delta = -theta); this package runs all three on the same kernels.
Deliberate differences:
  * aff_scan_forward is always exact (the reference's default repair=0 may
    not be) and does not build the reference's piecewise-affine chunk maps
    (:26-141): it runs the speculative segment forward (lead-ins from
    r(theta) = gamma*theta + delta, all segments at once, resynchronising
    fix-up; lifb_aff_scan_fwd).  `stats` reports what that path did
    ("segments", "lead_in") with repair_iters = 0.  C, K, BN, BNc, BNr are
    accepted; T % C == 0 and 0 <= gamma <= 1 are checked as the reference
    asserts them.
  * LIFAffineFn's adjoint is one fp32 reverse sweep per neuron instead of
    reverse_affine_scan's Hillis-Steele passes over [T, N].  When the forward
    is one streaming pass (mode "serial", or "scan" at lengths where the scan
    is that pass) the layer saves V (the potentials before the reset) instead
    of I and U, and the adjoint sweep reads V and gS once and accumulates the
    beta, gamma and delta sums in fp64 as it goes (lifb_aff_adjoint_v: 12 B
    per neuron-step for the whole backward); otherwise it saves I, u0, U and
    runs the adjoint and one fused parameter pass
    (lifb_aff_param_grad_partials).
  * reverse_affine_scan runs lifb_reverse_linear_scan (fp32, in order) for
    [T] and [T, ...] inputs.
"""
from __future__ import annotations

import torch

from . import _lib
from . import lifscan as L
from ._lib import check, ptr, stream_of

__all__ = ["aff_serial_forward", "aff_scan_forward", "reverse_affine_scan", "aff_adjoint", "aff_param_grads",
           "aff_serial_forward_v", "aff_adjoint_v", "LIFAffineFn", "lif_affine", "AFF_LEAD"]

# Lead-in rows of the speculative affine forward.  gamma < 1 contracts the
# state difference at every spike (gamma = 0 forgets the start at the first
# one); gamma = 1 (the soft reset) forgets only as fast as beta^t rounds it
# away, which needs about 1500-3000 rows at beta = 0.99.
AFF_LEAD = 8192


def _check_gamma(gamma):
    if not 0.0 <= float(gamma) <= 1.0:
        raise AssertionError(f"gamma must be in [0, 1], got {gamma}")


def aff_serial_forward(I, beta, theta, gamma, delta, u0, BN=32):
    """lifscan/triton_affine.py:158-162 -> (U, S): one pass of
    v = beta*u + x, s = v >= theta, u = s ? gamma*v + delta : v (fp32, no FMA)."""
    I, u0, T, N = L._prep_fwd(I, u0)
    U = torch.empty_like(I)
    S = torch.empty_like(I)
    lib = _lib.load()
    with torch.cuda.device(I.device):
        check(lib.lifb_aff_serial_fwd(ptr(I), ptr(u0), ptr(U), ptr(S), T, N, float(beta), float(theta),
                                      float(gamma), float(delta), stream_of(I)), "aff_serial_forward")
    return U, S


def aff_scan_forward(I, beta, theta, gamma, delta, u0, C=128, K=32, BN=16, BNc=16, BNr=32, repair=0, stats=None):
    """lifscan/triton_affine.py:165-199 -> (U, S), bit-identical to
    aff_serial_forward."""
    # the reference's asserts (triton_affine.py:167) come before any device work
    T = I.shape[0] if I.dim() == 2 else -1
    C = int(C)
    if T >= 0 and (C <= 0 or T % C):
        raise AssertionError(f"T={T} must be a multiple of C={C}")
    _check_gamma(gamma)
    I, u0, T, N = L._prep_fwd(I, u0)
    U = torch.empty_like(I)
    S = torch.empty_like(I)
    Lseg, _ = L.spec_segment(T, N)
    W = min(AFF_LEAD, Lseg) if Lseg < T else 0
    if stats is not None:
        stats.update(repair_iters=0, segments=T // Lseg if T else 0, lead_in=W)
    if T == 0 or N == 0:
        return U, S
    lib = _lib.load()
    with torch.cuda.device(I.device):
        nb = lib.lifb_scan_fwd_spec_workspace_bytes(T, N, Lseg) if Lseg < T else 0
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=I.device)
        check(lib.lifb_aff_scan_fwd(ptr(I), ptr(u0), ptr(U), ptr(S), T, N, float(beta), float(theta),
                                    float(gamma), float(delta), Lseg, W, ptr(ws), nb, stream_of(I)),
              "aff_scan_forward")
    return U, S


def reverse_affine_scan(a, b):
    """lifscan/triton_affine.py:202-211: lam_t = a_t * lam_{t+1} + b_t,
    lam_T = 0, along dim 0 of a [T, ...] CUDA fp32 tensor pair."""
    if a.shape != b.shape or a.dim() < 1:
        raise ValueError(f"a and b must have the same [T, ...] shape, got {tuple(a.shape)}, {tuple(b.shape)}")
    T = a.shape[0]
    N = 1
    for d in a.shape[1:]:
        N *= d
    A = L._cuda_f32("a", a.reshape(T, N))
    B = L._cuda_f32("b", b.reshape(T, N))
    out = torch.empty_like(A)
    lib = _lib.load()
    with torch.cuda.device(A.device):
        check(lib.lifb_reverse_linear_scan(ptr(A), ptr(B), ptr(out), T, N, stream_of(A)), "reverse_affine_scan")
    return out.reshape(a.shape)


def aff_adjoint(I, u0, U, gS, beta, theta, gamma, alpha=4.0):
    """lam = dL/dv of the affine-reset forward (I, u0) -> U under upstream
    gradient gS on S (detached spike), as LIFAffineFn.backward forms it
    (triton_affine.py:230-238)."""
    I, u0, T, N = L._prep_fwd(I, u0)
    U = L._cuda_f32("U", U, (T, N))
    gS = L._cuda_f32("gS", gS, (T, N))
    Lam = torch.empty_like(I)
    lib = _lib.load()
    with torch.cuda.device(I.device):
        check(lib.lifb_aff_adjoint(ptr(I), ptr(u0), ptr(U), ptr(gS), ptr(Lam), T, N, float(beta), float(theta),
                                   float(alpha), float(gamma), stream_of(I)), "aff_adjoint")
    return Lam


def aff_param_grads(I, u0, U, gS, Lam, beta, theta, alpha=4.0):
    """(dL/dbeta, dL/dgamma, dL/ddelta) as 0-d fp32 tensors
    (triton_affine.py:236-237): sum lam*u_{t-1}, sum S*V*beta*lam_{t+1},
    sum S*beta*lam_{t+1}; fp64 partial sums."""
    I, u0, T, N = L._prep_fwd(I, u0)
    U = L._cuda_f32("U", U, (T, N))
    gS = L._cuda_f32("gS", gS, (T, N))
    Lam = L._cuda_f32("Lam", Lam, (T, N))
    lib = _lib.load()
    M = max(lib.lifb_param_grad_chunks(T, N), 1)
    part = torch.zeros(4, M, N, dtype=torch.float64, device=I.device)
    with torch.cuda.device(I.device):
        check(lib.lifb_aff_param_grad_partials(ptr(I), ptr(u0), ptr(U), ptr(gS), ptr(Lam), ptr(part), T, N,
                                               float(beta), float(theta), float(alpha), M, stream_of(I)),
              "aff_param_grads")
    g = part.sum(dim=(1, 2)).to(torch.float32)
    return g[0], g[3], g[2]


def aff_serial_forward_v(I, beta, theta, gamma, delta, u0):
    """The serial affine forward returning (V, S): V[t] = v_t =
    fl(fl(beta*u_{t-1}) + x_t), the potential before the reset
    (lifb_aff_serial_fwd_v)."""
    I, u0, T, N = L._prep_fwd(I, u0)
    V = torch.empty_like(I)
    S = torch.empty_like(I)
    lib = _lib.load()
    with torch.cuda.device(I.device):
        check(lib.lifb_aff_serial_fwd_v(ptr(I), ptr(u0), ptr(V), ptr(S), T, N, float(beta), float(theta),
                                        float(gamma), float(delta), stream_of(I)), "aff_serial_forward_v")
    return V, S


def aff_adjoint_v(V, u0, gS, beta, theta, gamma, delta, alpha=4.0, param_grads=True):
    """lam = dL/dv from V (aff_serial_forward_v's output) and gS, and with
    param_grads the 0-d fp32 (dL/dbeta, dL/dgamma, dL/ddelta) of the same
    sweep -> (Lam, (d_beta, d_gamma, d_delta) or None)."""
    if V.dim() != 2:
        raise ValueError(f"V must be [T, N], got shape {tuple(V.shape)}")
    V = L._cuda_f32("V", V)
    T, N = V.shape
    u0 = L._cuda_f32("u0", u0, (N,))
    gS = L._cuda_f32("gS", gS, (T, N))
    Lam = torch.empty_like(V)
    # every entry is written by the sweep (no clearing launch needed)
    sums = torch.empty(3, N, dtype=torch.float64, device=V.device) if param_grads else None
    lib = _lib.load()
    with torch.cuda.device(V.device):
        check(lib.lifb_aff_adjoint_v(ptr(V), ptr(u0), ptr(gS), ptr(Lam), ptr(sums) if param_grads else None, T, N,
                                     float(beta), float(theta), float(alpha), float(gamma), float(delta),
                                     stream_of(V)), "aff_adjoint_v")
    if not param_grads:
        return Lam, None
    g = sums.sum(dim=1).to(torch.float32)
    return Lam, (g[0], g[1], g[2])


class LIFAffineFn(torch.autograd.Function):
    """lifscan/triton_affine.py:214-242: affine-reset LIF; grads w.r.t. I, u0,
    beta, gamma, delta (detached reset, sigmoid surrogate)."""

    @staticmethod
    def forward(ctx, I, u0, beta, gamma, delta, theta, alpha, mode, C, K):
        b, g, dl, th = L._host_scalars(beta, gamma, delta, theta)
        I = I.contiguous()
        T, N = I.shape
        ctx.cfg = (b, g, dl, th, alpha)
        if mode == "scan":
            if int(C) <= 0 or T % int(C):
                raise AssertionError(f"T={T} must be a multiple of C={C}")
            _check_gamma(g)
        ctx.vpath = L._single_pass(T, N, mode)
        if ctx.vpath:
            # one streaming pass: save V (same bytes as U) and let the adjoint
            # read V and gS only, with the parameter sums in the same sweep
            V, S = aff_serial_forward_v(I, b, th, g, dl, u0)
            ctx.save_for_backward(V, u0)
            return S
        if mode == "scan":
            U, S = aff_scan_forward(I, b, th, g, dl, u0, C=C, K=K)
        else:
            U, S = aff_serial_forward(I, b, th, g, dl, u0)
        ctx.save_for_backward(I, u0, U)
        return S

    @staticmethod
    def backward(ctx, gS):
        b, g, dl, th, alpha = ctx.cfg
        gS = gS.contiguous()
        need = ctx.needs_input_grad
        want_params = need[2] or need[3] or need[4]
        d_beta = d_gamma = d_delta = None
        if ctx.vpath:
            V, u0 = ctx.saved_tensors
            lam, pg = aff_adjoint_v(V, u0, gS, b, th, g, dl, alpha, param_grads=want_params)
            if want_params:
                d_beta, d_gamma, d_delta = pg
            _lib.poll_device("lif_affine backward")
            return (lam, b * lam[0], d_beta if need[2] else None, d_gamma if need[3] else None,
                    d_delta if need[4] else None, None, None, None, None, None)
        I, u0, U = ctx.saved_tensors
        # S is this layer's own output: the kernels recompute it from U and I
        lam = aff_adjoint(I, u0, U, gS, b, th, g, alpha)
        if want_params:
            d_beta, d_gamma, d_delta = aff_param_grads(I, u0, U, gS, lam, b, th, alpha)
        # parameters passed as Python numbers get no gradient
        _lib.poll_device("lif_affine backward")
        return (lam, b * lam[0], d_beta if need[2] else None, d_gamma if need[3] else None,
                d_delta if need[4] else None, None, None, None, None, None)


def lif_affine(I, u0, beta, gamma, delta, theta=1.0, alpha=4.0, mode="scan", C=128, K=32):
    """lifscan/triton_affine.py:245-246."""
    return LIFAffineFn.apply(I, u0, beta, gamma, delta, theta, alpha, mode, C, K)
