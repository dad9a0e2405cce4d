"""Drop-in mirror of the reference's `lifscan.triton_soft` (soft-reset LIF,
subtractive reset u <- v - theta) on B200 kernels.

    from hard_resets_compose_b200 import soft as S     # was: from lifscan import triton_soft as S
    U, Sp = S.soft_scan_forward(I, beta, 1.0, u0, C=32, K=16, repair=10**6)

Same names, arguments and return values as lifscan/triton_soft.py.
Deliberate differences:
  * soft_scan_forward is always exact (the reference's default repair=0 may
    not be) and does not build the reference's interval maps (:21-104): it
    runs the speculative segment forward (lead-ins, all segments at once,
    resynchronising fix-up; lifb_soft_scan_fwd).  `stats` reports what that
    path did ("segments", "lead_in") with repair_iters = 0; the reference's
    map statistics do not exist here.  C, K, BN, nw, BNc, BNr are accepted
    and ignored.
  * soft_adjoint_fft computes the same detached adjoint (lam_t = b_t +
    beta*lam_{t+1}) by the fp32 reverse sweep instead of a float64 FFT
    (within the 1e-5 gradient bar).
"""
from __future__ import annotations

import torch

from . import _lib
from . import lifscan as L
from ._lib import check, ptr, stream_of

__all__ = ["soft_serial_forward", "soft_serial_forward_tiled", "soft_scan_forward", "soft_adjoint_fft",
           "SOFT_LEAD"]

# Lead-in rows of the speculative soft forward: a soft reset forgets its start
# only as fast as beta^t rounds the difference away, so it needs longer
# lead-ins than the hard reset (about 1500-3000 rows at beta = 0.99).
SOFT_LEAD = 8192


def soft_serial_forward(I, beta, theta, u0, BN=32):
    """lifscan/triton_soft.py:168-172 -> (U, S)."""
    return L.soft_serial_forward(I, beta, theta, u0)


def soft_serial_forward_tiled(I, beta, theta, u0, BN=32, D=8, num_warps=1):
    """lifscan/triton_soft.py:250-254 (same results as soft_serial_forward)."""
    return L.soft_serial_forward(I, beta, theta, u0)


def soft_scan_forward(I, beta, theta, u0, C=32, K=16, BN=16, nw=1, BNc=16, BNr=32, repair=0, stats=None):
    """lifscan/triton_soft.py:175-211 -> (U, S), bit-identical to the serial
    soft recurrence."""
    I, u0, T, N = L._prep_fwd(I, u0)
    U = torch.empty_like(I)
    S = torch.empty_like(I)
    Lseg, W = L.spec_segment(T, N)
    W = min(SOFT_LEAD, Lseg) if Lseg < T else 0
    if stats is not None:
        stats.update(repair_iters=0, segments=T // Lseg if T else 0, lead_in=W)
    if T == 0 or N == 0:
        return U, S
    lib = _lib.load()
    with torch.cuda.device(I.device):
        nb = lib.lifb_scan_fwd_spec_workspace_bytes(T, N, Lseg) if Lseg < T else 0
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=I.device)
        check(lib.lifb_soft_scan_fwd(ptr(I), ptr(u0), ptr(U), ptr(S), T, N, float(beta), float(theta), Lseg, W,
                                     ptr(ws), nb, stream_of(I)), "soft_scan_forward")
    return U, S


def soft_adjoint_fft(V, gS, beta, theta, alpha=4.0):
    """lifscan/triton_soft.py:214-222: lam_t = b_t + beta*lam_{t+1},
    b_t = gS_t * sigma'(V_t - theta) (detached soft reset), V the pre-reset
    potentials."""
    if V.dim() != 2:
        raise ValueError(f"V must be [T, N], got shape {tuple(V.shape)}")
    V = L._cuda_f32("V", V)
    T, N = V.shape
    gS = L._cuda_f32("gS", gS, (T, N))
    Lam = torch.empty_like(V)
    lib = _lib.load()
    with torch.cuda.device(V.device):
        check(lib.lifb_soft_adjoint_v(ptr(V), ptr(gS), ptr(Lam), T, N, float(beta), float(theta), float(alpha),
                                      stream_of(V)), "soft_adjoint_fft")
    return Lam
