"""Drop-in mirror of the reference's `lifscan.triton_alif` (adaptive-threshold
LIF: state (u, w), threshold theta0 + w, w <- rho*w + q*s) on B200 kernels.

    from hard_resets_compose_b200 import alif as A     # was: from lifscan import triton_alif as A
    U, W, S = A.alif_serial_forward(I, 0.95, 0.995, 0.9, 1.0, 0.0, u0, w0)
    S, U, W = A.alif(I, u0, w0, beta, rho, q)           # grads for I, u0, w0, beta, rho, q, theta0

Same names, arguments and return values as lifscan/triton_alif.py.
Deliberate differences:
  * alif_scan_forward is always exact (the reference's default repair=0 may
    not be) and does not build the reference's box-restricted chunk maps
    (:95-253): it runs speculative segments (lead-ins of ALIF_LEAD rows
    started from (u_r, Wpred) where the prediction is given, all segments at
    once, then a fix-up that redoes a segment from its predecessor's true end
    until the (u, w, s) rows agree bit for bit; lifb_alif_scan_fwd).  Wpred
    only seeds the lead-ins, so any prediction, however bad, gives the same
    result; dw, K1, K2 and the Triton launch knobs are accepted and ignored.
    `stats` reports "segments" and "lead_in" with repair_iters = 0; `phases`
    receives the whole call's GPU time under "scan".
  * alif_backward's "scan" composes the chunk maps of the (lv, lw) pair
    (upper-triangular 2x2 per step), carries them and replays every chunk,
    over chunks of the B200 policy's length (lifscan.scan_chunk_bwd, at least
    ALIF_MIN_CHUNK rows: one chunk when N fills the GPU); it keeps the
    reference's argument checks
    (T % C == 0, C % D == 0).  The serial modes run one reverse sweep.
  * ALIFFn does not save S (its own output, recomputed bit for bit from U, W
    and I) and sums its parameter gradients in fp64 inside the same reverse
    sweep (lifb_alif_bwd with param_sums), without writing LW.
"""
from __future__ import annotations

import torch

from . import _lib
from . import lifscan as L
from ._lib import check, ptr, stream_of

__all__ = ["alif_fwd_cfg", "alif_serial_forward", "alif_warm_predict", "alif_scan_forward", "alif_backward",
           "ALIFFn", "alif", "ALIF_LEAD"]

# Lead-in rows of the speculative ALIF forward.  The adaptation w forgets its
# start only as fast as rho^t shrinks the difference below an ulp (about 3000
# rows at rho = 0.995), and two fp32 trajectories an ulp apart then merge only
# when fl(rho*w) rounds them together.  Measured at T = 2^18, N = 1024,
# rho = 0.995 (segments of 16384 rows): 8192-row lead-ins land on the exact
# state for 98% of the neurons and the fix-up of the rest costs 1 ms; 16384
# rows land on it for 99.99% (1.43 ms for the scan, 5.4 ms serial).  A warm-up
# prediction of w changes neither figure.
ALIF_LEAD = 16384


def _params(beta, rho, q, theta0, u_r):
    return tuple(float(v) for v in (beta, rho, q, theta0, u_r))


def _prep(I, u0, w0):
    I, u0, T, N = L._prep_fwd(I, u0)
    w0 = L._cuda_f32("w0", w0, (N,))
    if w0.device != I.device:
        raise ValueError("I and w0 must be on the same device")
    return I, u0, w0, T, N


def alif_fwd_cfg(N):
    """lifscan/triton_alif.py:255-260 (Triton launch shape; kept for signature
    compatibility, ignored by this implementation)."""
    if N <= 8:
        return 16, 16, 1
    if N <= 64:
        return 16, 4, 1
    if N <= 4096:
        return 32, 32, 1
    return 128, 8, 1


def alif_serial_forward(I, beta, rho, q, theta0, u_r, u0, w0, BN=32, D=0, num_warps=1):
    """lifscan/triton_alif.py:263-273 -> (U, W, S): one pass of the ALIF
    recurrence (fp32, no FMA).  D, BN, num_warps are accepted and ignored."""
    I, u0, w0, T, N = _prep(I, u0, w0)
    U = torch.empty_like(I)
    W = torch.empty_like(I)
    S = torch.empty_like(I)
    lib = _lib.load()
    with torch.cuda.device(I.device):
        check(lib.lifb_alif_serial_fwd(ptr(I), ptr(u0), ptr(w0), ptr(U), ptr(W), ptr(S), T, N,
                                       *_params(beta, rho, q, theta0, u_r), stream_of(I)), "alif_serial_forward")
    return U, W, S


def alif_warm_predict(I, beta, rho, q, theta0, u_r, u0, w0, C, Wn=4, u_init=0.0, w_init=0.0, BN=32, UI=None,
                      WI=None):
    """lifscan/triton_alif.py:276-285 -> WP [T//C, N]: the adaptation at the
    entry of every chunk of C rows, predicted by simulating the Wn chunks
    before it from (u_init, w_init), or from the chunk-entry states (UI, WI)
    of e.g. a previous iterate; from (u0, w0) when the warm-up reaches row 0."""
    I, u0, w0, T, N = _prep(I, u0, w0)
    C = int(C)
    if C <= 0 or T % C:
        raise ValueError(f"T={T} must be a multiple of C={C}")
    if (UI is None) != (WI is None):
        raise ValueError("UI and WI go together")
    M = T // C
    if UI is not None:
        UI = L._cuda_f32("UI", UI, (M, N))
        WI = L._cuda_f32("WI", WI, (M, N))
    WP = torch.empty(M, N, device=I.device)
    lib = _lib.load()
    with torch.cuda.device(I.device):
        check(lib.lifb_alif_warm_predict(ptr(I), ptr(u0), ptr(w0), ptr(WP), ptr(UI) if UI is not None else None,
                                         ptr(WI) if WI is not None else None, T, N, C, int(Wn), float(u_init),
                                         float(w_init), *_params(beta, rho, q, theta0, u_r), stream_of(I)),
              "alif_warm_predict")
    return WP


def alif_scan_forward(I, beta, rho, q, theta0, u_r, u0, w0, Wpred, dw, C=128, K1=16, K2=32, BN=16, nw=1, BNc=1,
                      BNr=32, D=4, repair=0, stats=None, phases=None):
    """lifscan/triton_alif.py:301-363 -> (U, W, S), bit-identical to
    alif_serial_forward.  Wpred [T//C, N] (or None) seeds the lead-ins."""
    # the reference's assert (triton_alif.py:308) comes before any device work
    T = I.shape[0] if I.dim() == 2 else -1
    C, D = int(C), int(D)
    if T >= 0 and (C <= 0 or D <= 0 or T % C or C % D):
        raise AssertionError(f"T={T} must be a multiple of C={C}, and C of D={D}")
    I, u0, w0, T, N = _prep(I, u0, w0)
    if Wpred is not None:
        Wpred = L._cuda_f32("Wpred", Wpred, (T // C, N))
    U = torch.empty_like(I)
    W = torch.empty_like(I)
    S = torch.empty_like(I)
    Lseg, _ = L.spec_segment(T, N)
    lead = min(ALIF_LEAD, Lseg) if Lseg < T else 0
    if stats is not None:
        stats.update(repair_iters=0, segments=T // Lseg if T else 0, lead_in=lead)
    if T == 0 or N == 0:
        return U, W, S
    lib = _lib.load()
    with torch.cuda.device(I.device):
        nb = lib.lifb_alif_scan_fwd_workspace_bytes(T, N, Lseg) if Lseg < T else 0
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=I.device)
        if phases is not None:
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(torch.cuda.current_stream(I.device))
        check(lib.lifb_alif_scan_fwd(ptr(I), ptr(u0), ptr(w0), ptr(U), ptr(W), ptr(S), T, N,
                                     *_params(beta, rho, q, theta0, u_r), Lseg, lead,
                                     ptr(Wpred) if Wpred is not None else None, C, ptr(ws), nb, stream_of(I)),
              "alif_scan_forward")
        if phases is not None:
            e1.record(torch.cuda.current_stream(I.device))
            e1.synchronize()
            phases["scan"] = e0.elapsed_time(e1)
    return U, W, S


# Shortest chunk of the two-level ALIF adjoint: the carry runs over the T/C
# chunks one after another, so very short chunks move the time into it
# (measured T = 4096, N = 8: 1-row chunks 1.72 ms against 0.38 ms for the one
# sweep).
ALIF_MIN_CHUNK = 256


def _alif_chunk(T, N):
    """Chunk length of the two-level ALIF adjoint: lifscan's adjoint policy
    (scan_chunk_bwd), doubled while it divides T until ALIF_MIN_CHUNK rows."""
    C = L.scan_chunk_bwd(T, N)
    while C < ALIF_MIN_CHUNK and C < T and T % (2 * C) == 0:
        C *= 2
    return C


def _alif_bwd(I, u0, w0, U, W, S, GS, beta, rho, q, theta0, alpha, want_lw, want_params, chunked=False):
    """(LV, LW or None, dL/dw0 or None, param sums [4, M, N] fp64 or None);
    chunked: over T/C chunks of the B200 policy's length (lifb_alif_bwd_scan)."""
    I, u0, w0, T, N = _prep(I, u0, w0)
    U = L._cuda_f32("U", U, (T, N))
    W = L._cuda_f32("W", W, (T, N))
    if S is not None:
        S = L._cuda_f32("S", S, (T, N))
    GS = L._cuda_f32("GS", GS, (T, N))
    C = _alif_chunk(T, N) if chunked and T > 0 else max(T, 1)
    M = T // C if T else 1
    LV = torch.empty_like(I)
    LW = torch.empty_like(I) if want_lw else None
    lwm1 = torch.empty(N, device=I.device) if want_params else None
    sums = torch.zeros(4, M, N, dtype=torch.float64, device=I.device) if want_params else None
    lib = _lib.load()
    o = lambda t: ptr(t) if t is not None else None  # noqa: E731
    with torch.cuda.device(I.device):
        nb = lib.lifb_alif_bwd_scan_workspace_bytes(T, N, C) if M > 1 else 0
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=I.device)
        check(lib.lifb_alif_bwd_scan(ptr(I), ptr(u0), ptr(w0), ptr(U), ptr(W), o(S), ptr(GS), ptr(LV), o(LW),
                                     o(lwm1), o(sums), T, N, float(beta), float(rho), float(q), float(theta0),
                                     float(alpha), C, ptr(ws), nb, stream_of(I)), "alif_backward")
    return LV, LW, lwm1, sums


def alif_backward(I, U, W, S, GS, beta, rho, q, theta0, u0, w0, alpha=4.0, mode="scan", C=64, BN=32, D=4, nw=1):
    """lifscan/triton_alif.py:490-521 -> (LV, LW): LV[t] = dL/dv_t (= dL/dI_t),
    LW[t] = dL/dw_t, for a loss with dL/dS = GS (detached reset).  "scan"
    runs the two-level form over chunks of the B200 policy's length (the
    reference's C and D are checked, not used); the serial modes one sweep."""
    if mode not in ("scan", "serial", "serial_pf", "serial_tuned"):
        raise ValueError(f"unknown mode {mode!r}")
    if mode == "scan":
        T = I.shape[0]
        C, D = int(C), int(D)
        if C <= 0 or D <= 0 or T % C or C % D:
            raise AssertionError(f"T={T} must be a multiple of C={C}, and C of D={D}")
    LV, LW, _, _ = _alif_bwd(I, u0, w0, U, W, S, GS, beta, rho, q, theta0, alpha, True, False,
                             chunked=mode == "scan")
    return LV, LW


class ALIFFn(torch.autograd.Function):
    """lifscan/triton_alif.py:524-554: S = ALIF(I; u0, w0, beta, rho, q, theta0)
    with u_r fixed; returns (S, U, W) (U, W not differentiable); gradients for
    I, u0, w0, beta, rho, q, theta0."""

    @staticmethod
    def forward(ctx, I, u0, w0, beta, rho, q, theta0, u_r, alpha, fwd, bwd, Wpred, dw, C, Cb):
        b, r, qq, th = L._host_scalars(beta, rho, q, theta0)
        I = I.contiguous()
        if fwd == "serial":
            U, W, S = alif_serial_forward(I, b, r, qq, th, u_r, u0, w0)
        else:
            U, W, S = alif_scan_forward(I, b, r, qq, th, u_r, u0, w0, Wpred, dw, C=C)
        ctx.save_for_backward(I, u0, w0, U, W)
        ctx.c = (b, r, qq, th, alpha)
        ctx.bwd = bwd
        ctx.mark_non_differentiable(U, W)
        return S, U, W

    @staticmethod
    def backward(ctx, gS, gU, gW):
        I, u0, w0, U, W = ctx.saved_tensors
        b, r, qq, th, alpha = ctx.c
        need = ctx.needs_input_grad
        want = any(need[1:7])
        # S is this layer's own output: the sweep recomputes it from U, W, I
        LV, _, lwm1, sums = _alif_bwd(I, u0, w0, U, W, None, gS.contiguous(), b, r, qq, th, alpha, False, want,
                                      chunked=ctx.bwd == "scan")
        g = sums.sum(dim=(1, 2)).to(torch.float32) if want else None
        pick = lambda i, v: v if need[i] else None  # noqa: E731
        _lib.poll_device("alif backward")
        return (LV, pick(1, b * LV[0]), pick(2, lwm1), pick(3, g[0] if want else None),
                pick(4, g[1] if want else None), pick(5, g[2] if want else None), pick(6, g[3] if want else None),
                None, None, None, None, None, None, None, None)


def alif(I, u0, w0, beta, rho, q, theta0=1.0, u_r=0.0, alpha=4.0, fwd="serial", bwd="scan", Wpred=None, dw=None,
         C=128, Cb=64):
    """lifscan/triton_alif.py:557-560: differentiable ALIF layer; returns (S, U,
    W).  Parameters may be 0-d tensors (requires_grad) or floats."""
    t = lambda v: v if torch.is_tensor(v) else torch.tensor(float(v), device=I.device)  # noqa: E731
    return ALIFFn.apply(I, u0, w0, t(beta), t(rho), t(q), t(theta0), u_r, alpha, fwd, bwd, Wpred, dw, C, Cb)
