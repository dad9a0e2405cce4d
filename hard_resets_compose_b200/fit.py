"""Differentiable hard-reset LIF with gradients w.r.t. the neuron parameters
(beta, theta, u_r), for fitting neuron models to long recordings: the GPU
half of the reference's lifscan/fit.py:15-61 (`LIFParamFn`, `lif_param`).

Forward and backward run this package's kernels (serial, scan or auto
dispatch, as the reference); the parameter gradients are read off the same
adjoint lam_t = dL/dv_t by one fused pass (lifb_param_grad_partials):
    dL/dbeta  = sum_t lam_t u_{t-1}
    dL/dtheta = -sum_t gS_t sigma'(v_t - theta)      (detached reset)
    dL/du_r   = sum_t s_t beta lam_{t+1}
The reference's CPU prototype backend (`LIFParamFnCPU`, built on fast.py) is
not part of this package: there is no CPU path.
"""
from __future__ import annotations

import torch

from . import _lib
from . import lifscan as L
from ._lib import check, ptr, stream_of

__all__ = ["LIFParamFn", "lif_param", "param_grads", "LIFSoftFn", "lif_soft", "LIFSoftScanFn", "lif_soft_scan"]


def param_grads(I, u0, U, GS, Lam, beta, theta, alpha=4.0):
    """(dL/dbeta, dL/dtheta, dL/du_r) as 0-d fp32 tensors from a detached-reset
    adjoint Lam of the forward (I, u0) -> U with upstream gradient GS on S."""
    I, u0, T, N = L._prep_fwd(I, u0)
    U = L._cuda_f32("U", U, (T, N))
    GS = L._cuda_f32("GS", GS, (T, N))
    Lam = L._cuda_f32("Lam", Lam, (T, N))
    lib = _lib.load()
    M = max(lib.lifb_param_grad_chunks(T, N), 1)
    part = torch.zeros(3, M, N, dtype=torch.float64, device=I.device)
    with torch.cuda.device(I.device):
        check(lib.lifb_param_grad_partials(ptr(I), ptr(u0), ptr(U), ptr(GS), ptr(Lam), ptr(part), T, N, float(beta),
                                           float(theta), float(alpha), M, stream_of(I)), "param_grads")
    g = part.sum(dim=(1, 2)).to(torch.float32)
    return g[0], g[1], g[2]


class LIFParamFn(torch.autograd.Function):
    """lifscan/fit.py:15-47: spikes out; gradients for I, u0, beta, theta, u_r."""

    @staticmethod
    def forward(ctx, I, u0, beta, theta, u_r, alpha, fwd_mode, bwd_mode, K):
        b, th, ur = L._host_scalars(beta, theta, u_r)
        I = I.contiguous()
        if fwd_mode == "scan":
            U, S = L.scan_forward_auto(I, b, th, ur, u0, K=K)
        else:
            U, S = L.serial_forward_auto(I, b, th, ur, u0)
        ctx.save_for_backward(I, u0, U)
        ctx.cfg = (b, th, ur, alpha, bwd_mode)
        return S

    @staticmethod
    def backward(ctx, gS):
        I, u0, U = ctx.saved_tensors
        b, th, ur, alpha, bwd_mode = ctx.cfg
        gS = gS.contiguous()
        # S is this layer's own output (recomputed bit for bit) and GU is zero
        if bwd_mode == "scan":
            lam = L.scan_backward_auto(I, u0, U, None, gS, None, b, th, ur, alpha)
        else:
            lam = L.serial_backward_auto(I, u0, U, None, gS, None, b, th, ur, alpha)
        g_beta, g_theta, g_ur = param_grads(I, u0, U, gS, lam, b, th, alpha)
        _lib.poll_device("fitting layer backward")
        return lam, b * lam[0], g_beta, g_theta, g_ur, None, None, None, None


def lif_param(I, u0, beta, theta, u_r, alpha=4.0, mode="auto", K=16):
    """lifscan/fit.py:50-56."""
    T, N = I.shape
    if mode == "auto":
        fwd, bwd = L.auto_modes(N, T)
    else:
        fwd = bwd = mode
    return LIFParamFn.apply(I, u0, beta, theta, u_r, alpha, fwd, bwd, K)


def _soft_beta_grad(I, u0, U, gS, lam, beta, theta, alpha):
    """dL/dbeta = sum_t lam_t u_{t-1} (lifscan/fit.py:116, :149), the fused
    reduction of param_grads (its other two sums belong to the hard reset)."""
    g_beta, _, _ = param_grads(I, u0, U, gS, lam, beta, theta, alpha)
    return g_beta


def _soft_forward_v(ctx, I, u0, b, th):
    """The soft layers' single-pass forward: the soft reset is the affine reset
    with gamma = 1, delta = -theta (bit for bit), so the layer saves V and its
    backward is the affine V-path sweep, which also sums dL/dbeta."""
    from . import affine as A
    V, S = A.aff_serial_forward_v(I, b, th, 1.0, -th, u0)
    ctx.save_for_backward(V, u0)
    return S


def _soft_backward_v(ctx, gS, b, th, alpha, need_beta):
    """(dI, du0, dbeta or None) from V: lam_t = gS_t sigma'(v_t) + beta
    lam_{t+1} and dbeta = sum lam_t u_{t-1} in the same sweep."""
    from . import affine as A
    V, u0 = ctx.saved_tensors
    lam, pg = A.aff_adjoint_v(V, u0, gS.contiguous(), b, th, 1.0, -th, alpha, param_grads=need_beta)
    return lam, b * lam[0], pg[0] if need_beta else None


class LIFSoftFn(torch.autograd.Function):
    """lifscan/fit.py:93-117: soft-reset LIF, serial kernels; gradients for I, u0,
    beta.  The layer saves V (the potentials before the reset) and its backward
    reads V and gS once, dbeta included (12 + 12 B per neuron-step)."""

    @staticmethod
    def forward(ctx, I, u0, beta, theta, alpha):
        b, th = L._host_scalars(beta, theta)
        I = I.contiguous()
        ctx.cfg = (b, th, alpha)
        return _soft_forward_v(ctx, I, u0, b, th)

    @staticmethod
    def backward(ctx, gS):
        b, th, alpha = ctx.cfg
        dI, du0, db = _soft_backward_v(ctx, gS, b, th, alpha, ctx.needs_input_grad[2])
        _lib.poll_device("fitting layer backward")
        return dI, du0, db, None, None


def lif_soft(I, u0, beta, theta=1.0, alpha=4.0):
    """lifscan/fit.py:120-121."""
    return LIFSoftFn.apply(I, u0, beta, theta, alpha)


class LIFSoftScanFn(torch.autograd.Function):
    """lifscan/fit.py:124-150: soft-reset LIF with the exact soft scan (or serial)
    forward; gradients for I, u0, beta.  mode in {"serial", "scan"}."""

    @staticmethod
    def forward(ctx, I, u0, beta, theta, alpha, mode, C, K):
        from . import soft as TS
        b, th = L._host_scalars(beta, theta)
        I = I.contiguous()
        ctx.cfg = (b, th, alpha)
        T, N = I.shape
        ctx.vpath = L._single_pass(T, N, mode)
        if ctx.vpath:  # one streaming pass: save V (see LIFSoftFn)
            return _soft_forward_v(ctx, I, u0, b, th)
        if mode == "scan":
            U, S = TS.soft_scan_forward(I, b, th, u0, C=C, K=K)
        else:
            U, S = L.soft_serial_forward(I, b, th, u0)
        ctx.save_for_backward(I, u0, U)
        return S

    @staticmethod
    def backward(ctx, gS):
        b, th, alpha = ctx.cfg
        if ctx.vpath:
            dI, du0, db = _soft_backward_v(ctx, gS, b, th, alpha, ctx.needs_input_grad[2])
            _lib.poll_device("fitting layer backward")
            return dI, du0, db, None, None, None, None, None
        I, u0, U = ctx.saved_tensors
        gS = gS.contiguous()
        # both modes: the same adjoint (the reference's scan mode forms V and
        # convolves by FFT, its serial mode sweeps; one sweep from U and I here)
        lam = L.soft_serial_backward_auto(I, u0, U, gS, b, th, alpha)
        _lib.poll_device("fitting layer backward")
        return lam, b * lam[0], _soft_beta_grad(I, u0, U, gS, lam, b, th, alpha), None, None, None, None, None


def lif_soft_scan(I, u0, beta, theta=1.0, alpha=4.0, mode="scan", C=128, K=32):
    """lifscan/fit.py:153-154."""
    return LIFSoftScanFn.apply(I, u0, beta, theta, alpha, mode, C, K)
