"""Drop-in mirror of the reference's `lifscan.triton_lif` API on B200 kernels.

    from hard_resets_compose_b200 import lifscan as L     # was: from lifscan import triton_lif as L
    S = L.lif_tuned(I, u0, beta=0.9, mode="scan")

Same names, argument order, defaults and return values as
lifscan/triton_lif.py; every call runs hand-written sm_100a CUDA kernels
through the C ABI of liblifb.so (include/lifscan_b200.h).  Triton tuning
knobs (BN, nw, BNc, nwc, BNr, D, nwr, BNg, nwg, num_warps) are accepted and
ignored: launch shapes are chosen by the library for B200.

Conventions (lifscan/triton_lif.py:3): I is [T, N] fp32 on a CUDA device
(made contiguous here), u0 is [N] fp32, beta/theta/u_r/alpha are Python
floats used as fp32; outputs are new tensors like torch.empty_like(I); S is
fp32 in {0, 1}.

Deliberate difference (recorded in the design notes): the forward always
repairs to convergence, so U and S are bit-identical to the serial fp32
recurrence for every `repair` value; `repair` is accepted for signature
compatibility and stats['repair_iters'] reports the rounds actually run.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import check, ptr, stream_of

__all__ = [
    "serial_forward", "serial_backward", "serial_forward_tiled", "serial_backward_tiled",
    "serial_backward_tiled_pf", "serial_forward_auto", "serial_backward_auto",
    "scan_forward", "scan_backward", "scan_forward_tiled", "scan_forward_v2", "scan_forward_v3",
    "scan_forward_v4", "scan_backward_tiled", "scan_forward_auto", "scan_backward_auto",
    "state_bounds", "surrogate_grad", "_pick_C", "LIFTuned", "lif_tuned", "LIFFunction", "lif",
    "AUTO_FWD_MAX_N", "AUTO_FWD_MIN_T", "AUTO_BWD_MAX_N", "AUTO_BWD_MIN_T", "auto_modes",
    "LIFAuto", "lif_auto", "serial_fwd_cfg", "serial_bwd_cfg", "scan_chunk_fwd", "scan_chunk_bwd",
    "lif_tuned_host", "scan_forward_spec", "spec_segment", "serial_forward_v", "lif_backward_v",
    "soft_serial_forward", "soft_serial_backward", "soft_serial_backward_pf", "soft_serial_backward_auto",
    "soft_bwd_cfg", "block_leadin",
]

_CONVERGE = -1  # max_repair value meaning "repair until converged"


# ----------------------------------------------------------------------------- checks
def _cuda_f32(name, t, shape=None):
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor (this implementation has no CPU path)")
    if t.dtype != torch.float32:
        raise TypeError(f"{name} must be float32, got {t.dtype}")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
    return t.contiguous()


def _prep_fwd(I, u0):
    if I.dim() != 2:
        raise ValueError(f"I must be [T, N], got shape {tuple(I.shape)}")
    I = _cuda_f32("I", I)
    T, N = I.shape
    u0 = _cuda_f32("u0", u0, (N,))
    if u0.device != I.device:
        raise ValueError("I and u0 are on different devices")
    return I, u0, T, N


def _prep_bwd(I, u0, U, S, GS, GU):
    I, u0, T, N = _prep_fwd(I, u0)
    U = _cuda_f32("U", U, (T, N))
    S = None if S is None else _cuda_f32("S", S, (T, N))
    GS = _cuda_f32("GS", GS, (T, N))
    GU = None if GU is None else _cuda_f32("GU", GU, (T, N))
    return I, u0, U, S, GS, GU, T, N


def _host_scalars(*xs):
    """The kernels take neuron parameters by value: read every tensor among xs
    to the host in one copy (one device sync instead of one per parameter)."""
    ts = [x for x in xs if torch.is_tensor(x)]
    vals = iter(torch.stack([t.detach().reshape(()).to(torch.float32) for t in ts]).tolist() if ts else [])
    return tuple(next(vals) if torch.is_tensor(x) else float(x) for x in xs)


def _f(x):
    return float(x)


# ----------------------------------------------------------------------------- serial
def serial_forward(I, beta, theta, u_r, u0, BN=None):
    """Serial hard-reset LIF forward (lifscan/triton_lif.py:246-251) -> (U, S)."""
    I, u0, T, N = _prep_fwd(I, u0)
    U = torch.empty_like(I)
    S = torch.empty_like(I)
    L = _lib.load()
    with torch.cuda.device(I.device):
        check(L.lifb_serial_fwd(ptr(I), ptr(u0), ptr(U), ptr(S), T, N, _f(beta), _f(theta), _f(u_r),
                                stream_of(I)), "serial_forward")
    return U, S


def serial_backward(I, u0, U, S, GS, GU, beta, theta, u_r, alpha=4.0, detach=True, BN=None):
    """Serial adjoint (lifscan/triton_lif.py:254-259) -> Lam = dL/dv = dL/dI.
    GU may be None (zeros).  S may be None when it is the forward's own
    output: the spikes are then recomputed bit-exactly from U and I instead
    of being read."""
    I, u0, U, S, GS, GU, T, N = _prep_bwd(I, u0, U, S, GS, GU)
    Lam = torch.empty_like(I)
    L = _lib.load()
    with torch.cuda.device(I.device):
        check(L.lifb_serial_bwd(ptr(I), ptr(u0), ptr(U), ptr(S), ptr(GS), ptr(GU), ptr(Lam), T, N, _f(beta),
                                _f(theta), _f(u_r), _f(alpha), int(bool(detach)), stream_of(I)),
              "serial_backward")
    return Lam


def serial_forward_tiled(I, beta, theta, u_r, u0, BN=32, D=4, num_warps=1):
    """lifscan/triton_lif.py:460-466 (same results as serial_forward)."""
    return serial_forward(I, beta, theta, u_r, u0)


def serial_backward_tiled(I, u0, U, S, GS, GU, beta, theta, u_r, alpha=4.0, detach=True, BN=32, D=4,
                          num_warps=1):
    """lifscan/triton_lif.py:469-476."""
    return serial_backward(I, u0, U, S, GS, GU, beta, theta, u_r, alpha, detach)


def serial_backward_tiled_pf(I, u0, U, S, GS, GU, beta, theta, u_r, alpha=4.0, detach=True, BN=32, D=4,
                             num_warps=1):
    """lifscan/triton_lif.py:1130-1135."""
    return serial_backward(I, u0, U, S, GS, GU, beta, theta, u_r, alpha, detach)


def serial_fwd_cfg(N):
    """Kept for signature compatibility (lifscan/triton_lif.py:1213-1218); the
    B200 kernels choose their own tiles."""
    return 32, 16, 1


def serial_bwd_cfg(N):
    """Kept for signature compatibility (lifscan/triton_lif.py:1184-1189)."""
    return 32, 8, 1


def serial_forward_auto(I, beta, theta, u_r, u0):
    """lifscan/triton_lif.py:1221-1225."""
    return serial_forward(I, beta, theta, u_r, u0)


def serial_backward_auto(I, u0, U, S, GS, GU, beta, theta, u_r, alpha=4.0, detach=True):
    """lifscan/triton_lif.py:1199-1203."""
    return serial_backward(I, u0, U, S, GS, GU, beta, theta, u_r, alpha, detach)


# ----------------------------------------------------------------------------- scan forward
def _stats_buffer(dev, want):
    return torch.zeros(_lib.STATS_BYTES, dtype=torch.uint8, device=dev) if want else None


def _fill_stats(stats, buf, level):
    st = _lib.read_stats(buf)  # the host waits here anyway: fold in the device status
    _lib.check_device("scan stats")
    stats["repair_iters"] = int(st.repair_iters)
    n = max(int(st.n_maps), 1)
    stats["overflow_frac"] = float(st.n_overflow) / n
    stats["mean_pieces"] = float(st.sum_cnt) / n + 1.0
    if level == 3:
        stats["max_pieces"] = int(st.max_cnt) + 1
    else:
        ns = max(int(st.n_super), 1)
        stats["super_overflow_frac"] = float(st.n_super_overflow) / ns
        stats["super_mean_pieces"] = float(st.sum_super_cnt) / ns + 1.0
        stats["super_max_pieces"] = int(st.max_super_cnt) + 1


def scan_forward_v3(I, beta, theta, u_r, u0, C=64, K=16, BN=32, nw=1, BNc=16, nwc=1, BNr=32, D=8, nwr=1,
                    repair=0, stats=None):
    """Two-level exact scan (lifscan/triton_lif.py:782-817) -> (U, S).

    Envelope-pruned chunk maps of length C and capacity K, sequential carry,
    replay, and device-side repair to convergence."""
    I, u0, T, N = _prep_fwd(I, u0)
    C, K = int(C), int(K)
    if C <= 0 or T % C:
        raise ValueError(f"T={T} must be a positive multiple of C={C}")
    U = torch.empty_like(I)
    S = torch.empty_like(I)
    L = _lib.load()
    with torch.cuda.device(I.device):
        nb = L.lifb_scan_fwd_v3_workspace_bytes(T, N, C, K)
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=I.device)
        sb = _stats_buffer(I.device, stats is not None)
        check(L.lifb_scan_fwd_v3(ptr(I), ptr(u0), ptr(U), ptr(S), T, N, _f(beta), _f(theta), _f(u_r), C, K,
                                 _CONVERGE, ptr(ws), nb, ptr(sb), stream_of(I)), "scan_forward_v3")
        if stats is not None:
            _fill_stats(stats, sb, 3)
    return U, S


def scan_forward_v4(I, beta, theta, u_r, u0, C=64, G=16, K=16, K2=32, BN=32, nw=1, BNg=16, nwg=1, BNc=16,
                    nwc=1, BNr=32, D=8, nwr=1, repair=0, stats=None):
    """Three-level exact scan (lifscan/triton_lif.py:935-983) -> (U, S)."""
    I, u0, T, N = _prep_fwd(I, u0)
    C, G, K, K2 = int(C), int(G), int(K), int(K2)
    if C <= 0 or G <= 0 or T % (C * G):
        raise AssertionError("T must be divisible by C*G")
    U = torch.empty_like(I)
    S = torch.empty_like(I)
    L = _lib.load()
    with torch.cuda.device(I.device):
        nb = L.lifb_scan_fwd_v4_workspace_bytes(T, N, C, G, K, K2)
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=I.device)
        sb = _stats_buffer(I.device, stats is not None)
        check(L.lifb_scan_fwd_v4(ptr(I), ptr(u0), ptr(U), ptr(S), T, N, _f(beta), _f(theta), _f(u_r), C, G, K, K2,
                                 _CONVERGE, ptr(ws), nb, ptr(sb), stream_of(I)), "scan_forward_v4")
        if stats is not None:
            _fill_stats(stats, sb, 4)
    return U, S


def scan_forward(I, beta, theta, u_r, u0, C=64, K=16, BN=None, repair=0, stats=None):
    """Legacy entry (lifscan/triton_lif.py:262-295); runs the v3 algorithm,
    whose envelope bound is tighter than the legacy global bound.  Outputs are
    identical (both are exact); stats describe the v3 maps."""
    return scan_forward_v3(I, beta, theta, u_r, u0, C=C, K=K, repair=repair, stats=stats)


def scan_forward_tiled(I, beta, theta, u_r, u0, C=64, K=16, BN=128, BNr=32, D=4, nw=4, nwr=1, repair=0,
                       stats=None):
    """Legacy entry (lifscan/triton_lif.py:479-509); runs the v3 algorithm."""
    return scan_forward_v3(I, beta, theta, u_r, u0, C=C, K=K, repair=repair, stats=stats)


def scan_forward_v2(I, beta, theta, u_r, u0, C=64, K=16, BN=128, nw=4, STAGES=3, CSTAGES=1, BNr=32, D=4, nwr=1,
                    repair=0, stats=None, Imin=None):
    """Legacy entry (lifscan/triton_lif.py:609-642); runs the v3 algorithm."""
    return scan_forward_v3(I, beta, theta, u_r, u0, C=C, K=K, repair=repair, stats=stats)


def _pick_C(T, D=8):
    """lifscan/triton_lif.py:647-651: largest C in (256, ..., 8) with T % C == 0,
    C % D == 0 and C*C <= 4T."""
    for C in (256, 128, 64, 32, 16, 8):
        if T % C == 0 and C % D == 0 and C * C <= 4 * T:
            return C
    raise ValueError(f"T={T} needs a chunk length divisible by {D}")


# Chunk lengths of lif_tuned's scan mode on B200, chosen from CUDA-event
# timings of every path on a B200:
#  * forward: the single streaming pass (one chunk, C = T: the scan's replay
#    pass from u0) is faster than building maps at every width measured, from
#    N = 1024 x T = 2^20 (19 ms vs 34 ms for the map scan) to N = 16384 x
#    T = 1024, so the auto path uses it; scan_forward_v3/v4 called directly still
#    build and carry maps with the caller's C and K.
#  * adjoint: below N = 8192 the single pass is chain-bound, and long chunks
#    replayed in parallel from lam_end = 0 plus the tail fix-up (the detached
#    reset zeroes the carry at every spike) win: T = 2^20, N = 1024 in ~4 ms vs
#    43 ms.  Chunks are long (about 8 warps per SM in flight) so tails are rare.
SCAN_FWD_SERIAL_MIN_N = 0
SCAN_BWD_SERIAL_MIN_N = 8192


def _long_chunk(T, N, warps_per_sm=8, sms=148):
    """Largest power-of-two divisor C of T that still gives about
    warps_per_sm x sms (chunk, 32-neuron) warps."""
    want = max(1, -(-warps_per_sm * sms * 32 // max(N, 1)))
    C = T
    while C % 2 == 0 and T // C < want:
        C //= 2
    return C


def scan_chunk_fwd(T, N):
    """Chunk length of lif_tuned's scan forward on B200 (see above)."""
    return T if N >= SCAN_FWD_SERIAL_MIN_N else _pick_C(T, D=16)


def scan_chunk_bwd(T, N):
    """Chunk length of lif_tuned's scan backward on B200 (see above)."""
    return T if N >= SCAN_BWD_SERIAL_MIN_N else _long_chunk(T, N)


# Speculative segment forward (lifb_scan_fwd_spec): when N neurons alone
# cannot fill the GPU (N < SPEC_FILL, about 8 warps per SM), the sequence is
# cut into segments of SPEC_L rows (a power of two down to SPEC_MIN_L that
# divides T into at least two) started from SPEC_LEAD-row lead-ins and fixed
# up exactly.  Measured on B200 at N = 1024, x ~ N(0.02, 0.1^2), beta = 0.99:
# T = 2^20 takes 2.7 ms against 19.3 ms for the single pass, T = 2^17 0.55 ms
# against 2.4 ms; shorter segments or lead-ins below ~2048 rows lose time
# in the fix-up, longer lead-ins re-read more rows.
SPEC_FILL = 8 * 148 * 32
SPEC_L = 16384
SPEC_MIN_L = 4096
SPEC_LEAD = 4096


def spec_segment(T, N):
    """(L, W) of lif_tuned's scan forward on B200: L = T is the single pass."""
    if N >= SPEC_FILL:
        return T, 0
    L = SPEC_L
    while L >= SPEC_MIN_L and (T % L or T // L < 2):
        L //= 2
    if L < SPEC_MIN_L:
        return T, 0
    return L, min(SPEC_LEAD, L)


# Block-level lead-in forward for short sequences with few neurons
# (lifb_scan_fwd_spec with segments of BLOCK_L rows runs csrc/scan_block.cu):
# one CTA per 32-neuron slab holds all T rows on chip, each warp guesses its
# chunk's start with a W-row lead-in from u_r and replays it at once, and
# fix-up rounds replay the rare wrong guesses until they rejoin.  W must
# outlast the rows two trajectories of one neuron take to become identical,
# which grows like 1/(-ln beta) (the rows for beta^k to shrink a difference
# below one ulp: 24 ln 2 / -ln beta); 1.6 times that, in 64-row steps, is
# 256 rows at beta = 0.9, where the measured p99.9 is about 150 rows
# (config 1).  It pays while the chain W + L stays under half the single
# pass's T rows and the neurons alone cannot fill the GPU: measured on B200
# at T = 1024, beta = 0.9: N = 4096 16.4 us against 24.6 us for the single
# pass, N = 8192 27.7 against 25.8 us.
BLOCK_L = 64
BLOCK_MAX_N = 6144
BLOCK_MAX_T = 1536


def block_leadin(T, N, beta):
    """(L, W) of the block-level lead-in forward for this shape and beta, or
    (0, 0) when the single pass (or the long-sequence path) is the choice."""
    import math
    if not (0 < N <= BLOCK_MAX_N and N % 4 == 0 and 0 < T <= BLOCK_MAX_T and T % BLOCK_L == 0
            and T // BLOCK_L >= 2 and 0.0 < beta < 1.0):
        return 0, 0
    rows = 1.6 * 24.0 * math.log(2.0) / -math.log(beta)
    W = BLOCK_L * max(1, math.ceil(rows / BLOCK_L))
    if W + BLOCK_L > T // 2:
        return 0, 0
    return BLOCK_L, W


def scan_forward_spec(I, beta, theta, u_r, u0, L=None, W=None, halo=None):
    """Speculative segment forward (lifb_scan_fwd_spec) -> (U, S), identical to
    the serial recurrence; L = segment length (T % L == 0), W = lead-in rows
    (defaults: spec_segment).  halo [W_halo, N]: rows before row 0; u0 is then
    the (guessed) state before the halo and the result is exact for the state
    the halo leads to."""
    I, u0, T, N = _prep_fwd(I, u0)
    if halo is not None:
        halo = _cuda_f32("halo", halo)
        if halo.dim() != 2 or halo.shape[1] != N:
            raise ValueError(f"halo must be [W, {N}], got {tuple(halo.shape)}")
    U = torch.empty_like(I)
    S = torch.empty_like(I)
    if T == 0 or N == 0:
        return U, S
    Ld, Wd = spec_segment(T, N)
    L = Ld if L is None else int(L)
    W = Wd if W is None else int(W)
    if L <= 0 or T % L:
        raise ValueError(f"T={T} is not a multiple of the segment length L={L}")
    lib = _lib.load()
    with torch.cuda.device(I.device):
        nb = lib.lifb_scan_fwd_spec_workspace_bytes(T, N, L)
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=I.device)
        check(lib.lifb_scan_fwd_spec(ptr(I), ptr(u0), ptr(U), ptr(S), T, N, _f(beta), _f(theta), _f(u_r), L, W,
                                     ptr(halo), 0 if halo is None else halo.shape[0], ptr(ws), nb, stream_of(I)),
              "scan_forward_spec")
    return U, S


def scan_forward_auto(I, beta, theta, u_r, u0, K=16, repair=0):
    """lifscan/triton_lif.py:1228-1232 with a B200 path choice: the single
    streaming pass; the speculative segment forward when N is too small to
    fill the GPU and T is long (spec_segment); the block-level lead-in
    forward when T is short and N small (block_leadin).  Outputs are
    identical whichever runs (exact)."""
    T, N = I.shape
    if T > 0 and N > 0 and spec_segment(T, N)[0] < T:
        return scan_forward_spec(I, beta, theta, u_r, u0)
    Lb, Wb = block_leadin(T, N, float(beta))
    if Lb:
        return scan_forward_spec(I, beta, theta, u_r, u0, L=Lb, W=Wb)
    return scan_forward_v3(I, beta, theta, u_r, u0, C=scan_chunk_fwd(T, N), K=K, repair=repair)


# ----------------------------------------------------------------------------- scan backward
def scan_backward_tiled(I, u0, U, S, GS, GU, beta, theta, u_r, alpha=4.0, detach=True, C=64, BNr=32, D=4,
                        nwr=1):
    """Tiled affine-scan backward (lifscan/triton_lif.py:512-526) -> Lam.
    GU may be None (zeros); S may be None as for serial_backward."""
    I, u0, U, S, GS, GU, T, N = _prep_bwd(I, u0, U, S, GS, GU)
    C = int(C)
    if C <= 0 or T % C:
        raise ValueError(f"T={T} must be a positive multiple of C={C}")
    Lam = torch.empty_like(I)
    L = _lib.load()
    with torch.cuda.device(I.device):
        nb = L.lifb_scan_bwd_workspace_bytes(T, N, C)
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=I.device)
        check(L.lifb_scan_bwd(ptr(I), ptr(u0), ptr(U), ptr(S), ptr(GS), ptr(GU), ptr(Lam), T, N, _f(beta),
                              _f(theta), _f(u_r), _f(alpha), int(bool(detach)), C, ptr(ws), nb, stream_of(I)),
              "scan_backward_tiled")
    return Lam


def scan_backward(I, u0, U, S, GS, GU, beta, theta, u_r, alpha=4.0, detach=True, C=64, BN=None):
    """Legacy entry (lifscan/triton_lif.py:298-312)."""
    return scan_backward_tiled(I, u0, U, S, GS, GU, beta, theta, u_r, alpha, detach, C=C)


def scan_backward_auto(I, u0, U, S, GS, GU, beta, theta, u_r, alpha=4.0):
    """lifscan/triton_lif.py:1235-1239 with a B200 chunk choice (scan_chunk_bwd)."""
    T, N = I.shape
    return scan_backward_tiled(I, u0, U, S, GS, GU, beta, theta, u_r, alpha, C=scan_chunk_bwd(T, N))


# ----------------------------------------------------------------------------- helpers
def state_bounds(I, beta, theta, u_r, u0):
    """Loose global state bounds (lifscan/triton_lif.py:238-243); host helper,
    not on the kernel path."""
    Imin = I.min(0).values.clamp(max=0)
    base = torch.minimum(u0, torch.full_like(u0, u_r)).clamp(max=0)
    lo = base + (Imin / (1 - beta) if beta < 1 else I.clamp(max=0).sum(0))
    hi = torch.maximum(u0, torch.full_like(u0, max(theta, u_r)))
    return lo.contiguous(), hi.contiguous()


def surrogate_grad(x, alpha):
    """Derivative of sigmoid(alpha*x) (lifscan/fast.py:48-51)."""
    sg = torch.sigmoid(alpha * x)
    return alpha * sg * (1 - sg)


# ----------------------------------------------------------------------------- soft reset (serial)
def soft_serial_forward(I, beta, theta, u0, BN=32):
    """Soft-reset serial forward (lifscan/triton_lif.py:1072-1076) -> (U, S):
    u <- v - theta on a spike instead of u_r."""
    I, u0, T, N = _prep_fwd(I, u0)
    U = torch.empty_like(I)
    S = torch.empty_like(I)
    lib = _lib.load()
    with torch.cuda.device(I.device):
        check(lib.lifb_soft_serial_fwd(ptr(I), ptr(u0), ptr(U), ptr(S), T, N, _f(beta), _f(theta), stream_of(I)),
              "soft_serial_forward")
    return U, S


def soft_serial_backward(I, u0, U, GS, beta, theta, alpha=4.0, BN=32):
    """Soft-reset detached adjoint (lifscan/triton_lif.py:1079-1083) -> Lam."""
    I, u0, T, N = _prep_fwd(I, u0)
    U = _cuda_f32("U", U, (T, N))
    GS = _cuda_f32("GS", GS, (T, N))
    Lam = torch.empty_like(I)
    lib = _lib.load()
    with torch.cuda.device(I.device):
        check(lib.lifb_soft_serial_bwd(ptr(I), ptr(u0), ptr(U), ptr(GS), ptr(Lam), T, N, _f(beta), _f(theta),
                                       _f(alpha), stream_of(I)), "soft_serial_backward")
    return Lam


def soft_serial_backward_pf(I, u0, U, GS, beta, theta, alpha=4.0, BN=32, D=4, num_warps=1):
    """lifscan/triton_lif.py:1176-1180 (same results as soft_serial_backward)."""
    return soft_serial_backward(I, u0, U, GS, beta, theta, alpha)


def soft_bwd_cfg(N):
    """lifscan/triton_lif.py:1192-1196 (Triton launch shape; kept for signature
    compatibility, ignored by this implementation)."""
    if N <= 8:
        return 16, 8, 1
    if N <= 64:
        return 16, 4, 1
    if N <= 16384:
        return 64, 16, 1
    return 128, 4, 1


def soft_serial_backward_auto(I, u0, U, GS, beta, theta, alpha=4.0):
    """lifscan/triton_lif.py:1206-1210."""
    return soft_serial_backward(I, u0, U, GS, beta, theta, alpha)


# ----------------------------------------------------------------------------- V-saving layer path
def serial_forward_v(I, beta, theta, u_r, u0):
    """Serial forward that returns (V, S), V[t] = v_t = fl(fl(beta*u_{t-1}) + x_t),
    the potential before the reset (lifb_serial_fwd_v); S as serial_forward."""
    I, u0, T, N = _prep_fwd(I, u0)
    V = torch.empty_like(I)
    S = torch.empty_like(I)
    lib = _lib.load()
    with torch.cuda.device(I.device):
        check(lib.lifb_serial_fwd_v(ptr(I), ptr(u0), ptr(V), ptr(S), T, N, _f(beta), _f(theta), _f(u_r),
                                    stream_of(I)), "serial_forward_v")
    return V, S


def lif_backward_v(V, GS, beta, theta, alpha=4.0, C=None):
    """Detached-reset adjoint of lif_tuned from V and GS alone (lifb_lif_bwd_v)
    -> Lam = dL/dI; du0 = beta * Lam[0].  C = chunk length (default T)."""
    if V.dim() != 2:
        raise ValueError(f"V must be [T, N], got shape {tuple(V.shape)}")
    V = _cuda_f32("V", V)
    T, N = V.shape
    GS = _cuda_f32("GS", GS, (T, N))
    C = T if C is None else int(C)
    Lam = torch.empty_like(V)
    lib = _lib.load()
    with torch.cuda.device(V.device):
        nb = lib.lifb_lif_bwd_v_workspace_bytes(T, N, C) if C < T else 0
        ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=V.device)
        check(lib.lifb_lif_bwd_v(ptr(V), ptr(GS), ptr(Lam), T, N, _f(beta), _f(theta), _f(alpha), C, ptr(ws), nb,
                                 stream_of(V)), "lif_backward_v")
    return Lam


def _single_pass(T, N, mode):
    """True when lif_tuned's forward is the single streaming pass (where it
    saves V instead of U)."""
    return T > 0 and N > 0 and (mode == "serial" or spec_segment(T, N)[0] == T)


# ----------------------------------------------------------------------------- autograd layers
class LIFTuned(torch.autograd.Function):
    """Hard-reset LIF, detached reset, sigmoid surrogate (lifscan/triton_lif.py:654-683).
    mode in {"serial", "scan"}; returns spikes S [T, N]."""

    @staticmethod
    def forward(ctx, I, u0, beta, theta, u_r, alpha, mode, K, repair):
        I = I.contiguous()
        T, N = I.shape
        ctx.cfg = (beta, theta, u_r, alpha, mode)
        ctx.vpath = _single_pass(T, N, mode)
        if ctx.vpath:
            # the adjoint needs only v_t: save V (same bytes as U) and read
            # V and GS in the backward instead of I, U and GS
            V, S = serial_forward_v(I, beta, theta, u_r, u0)
            ctx.save_for_backward(V)
            return S
        if mode == "serial":
            U, S = serial_forward_auto(I, beta, theta, u_r, u0)
        else:
            U, S = scan_forward_auto(I, beta, theta, u_r, u0, K=K, repair=repair)
        ctx.save_for_backward(I, u0, U, S)
        return S

    @staticmethod
    def backward(ctx, gS):
        beta, theta, u_r, alpha, mode = ctx.cfg
        gS = gS.contiguous()
        if ctx.vpath:
            (V,) = ctx.saved_tensors
            T, N = V.shape
            Lam = lif_backward_v(V, gS, beta, theta, alpha, C=T if mode == "serial" else scan_chunk_bwd(T, N))
            _lib.poll_device("lif_tuned")
            return Lam, beta * Lam[0], None, None, None, None, None, None, None
        I, u0, U, S = ctx.saved_tensors
        # GU is identically zero on this path: pass None instead of materialising
        # zeros_like(gS); S is this layer's own forward output, so the kernels
        # recompute it bit-exactly from U and I instead of reading it (S=None).
        if mode == "serial":
            Lam = serial_backward_auto(I, u0, U, None, gS, None, beta, theta, u_r, alpha)
        else:
            Lam = scan_backward_auto(I, u0, U, None, gS, None, beta, theta, u_r, alpha)
        _lib.poll_device("lif_tuned")
        return Lam, beta * Lam[0], None, None, None, None, None, None, None


def lif_tuned(I, u0, beta=0.9, theta=1.0, u_r=0.0, alpha=4.0, mode="scan", K=16, repair=0):
    """lifscan/triton_lif.py:686-687."""
    return LIFTuned.apply(I, u0, beta, theta, u_r, alpha, mode, K, repair)


class LIFFunction(torch.autograd.Function):
    """Legacy layer (lifscan/triton_lif.py:315-339) with an explicit chunk length C."""

    @staticmethod
    def forward(ctx, I, u0, beta, theta, u_r, alpha, mode, C, K, repair):
        I = I.contiguous()
        if mode == "serial":
            U, S = serial_forward(I, beta, theta, u_r, u0)
        else:
            U, S = scan_forward(I, beta, theta, u_r, u0, C=C, K=K, repair=repair)
        ctx.save_for_backward(I, u0, U, S)
        ctx.cfg = (beta, theta, u_r, alpha, mode, C)
        return S

    @staticmethod
    def backward(ctx, gS):
        I, u0, U, S = ctx.saved_tensors
        beta, theta, u_r, alpha, mode, C = ctx.cfg
        gS = gS.contiguous()
        if mode == "serial":
            Lam = serial_backward(I, u0, U, None, gS, None, beta, theta, u_r, alpha)
        else:
            Lam = scan_backward(I, u0, U, None, gS, None, beta, theta, u_r, alpha, C=C)
        _lib.poll_device("lif")
        return Lam, beta * Lam[0], None, None, None, None, None, None, None, None


def lif(I, u0, beta=0.9, theta=1.0, u_r=0.0, alpha=4.0, mode="scan", C=64, K=16, repair=0):
    """lifscan/triton_lif.py:342-343."""
    return LIFFunction.apply(I, u0, beta, theta, u_r, alpha, mode, C, K, repair)


# ----------------------------------------------------------------------------- auto dispatch
# Scan only where the serial recurrence cannot fill the GPU (lifscan/triton_lif.py:986-1000).
# The reference calibrated these on an RTX 5090; these values are B200's: the serial
# kernels saturate HBM once ~5k independent recurrences are in flight, so time
# parallelism pays only below that width (and only for long enough T).
AUTO_FWD_MAX_N = 4096
AUTO_FWD_MIN_T = 4096
AUTO_BWD_MAX_N = 4096
AUTO_BWD_MIN_T = 2048


def auto_modes(N, T):
    """lifscan/triton_lif.py:997-1000 -> (fwd_mode, bwd_mode)."""
    fwd = "scan" if (N <= AUTO_FWD_MAX_N and T >= AUTO_FWD_MIN_T) else "serial"
    bwd = "scan" if (N <= AUTO_BWD_MAX_N and T >= AUTO_BWD_MIN_T) else "serial"
    return fwd, bwd


class LIFAuto(torch.autograd.Function):
    """lifscan/triton_lif.py:1003-1026."""

    @staticmethod
    def forward(ctx, I, u0, beta, theta, u_r, alpha, K, repair, fwd_mode, bwd_mode):
        I = I.contiguous()
        if fwd_mode == "scan":
            U, S = scan_forward_auto(I, beta, theta, u_r, u0, K=K, repair=repair)
        else:
            U, S = serial_forward_auto(I, beta, theta, u_r, u0)
        ctx.save_for_backward(I, u0, U, S)
        ctx.cfg = (beta, theta, u_r, alpha, bwd_mode)
        return S

    @staticmethod
    def backward(ctx, gS):
        I, u0, U, S = ctx.saved_tensors
        beta, theta, u_r, alpha, bwd_mode = ctx.cfg
        gS = gS.contiguous()
        if bwd_mode == "scan":
            Lam = scan_backward_auto(I, u0, U, None, gS, None, beta, theta, u_r, alpha)
        else:
            Lam = serial_backward_auto(I, u0, U, None, gS, None, beta, theta, u_r, alpha)
        _lib.poll_device("lif_auto")
        return Lam, beta * Lam[0], None, None, None, None, None, None, None, None


def lif_auto(I, u0, beta=0.9, theta=1.0, u_r=0.0, alpha=4.0, K=16, repair=0):
    """lifscan/triton_lif.py:1029-1031."""
    fwd, bwd = auto_modes(I.shape[1], I.shape[0])
    return LIFAuto.apply(I, u0, beta, theta, u_r, alpha, K, repair, fwd, bwd)


# ----------------------------------------------------------------------------- host-resident tensors
def lif_tuned_host(I, GS, u0=None, beta=0.9, theta=1.0, u_r=0.0, alpha=4.0, block_n=None, device=None,
                   out=None, sync=True, block_t=None):
    """lif_tuned forward + backward for host (CPU) tensors, pipelined so
    host->device copies, compute and device->host copies overlap.  Returns
    (S, dI, du0) as CPU tensors (pinned); equivalent to S = lif_tuned(I, u0,
    ...); torch.autograd.backward(S, GS) with dI = I.grad and du0 = u0.grad.
    The pipeline runs over blocks of time rows (lifb_lif_fwd_bwd_host_rows:
    contiguous copies, block_t rows, default about 16 MiB per block) when N %
    4 == 0 and block_n is not given, else over blocks of block_n neurons
    (lifb_lif_fwd_bwd_host); both give the same bits.
    I and GS should be pinned for full overlap; `out` may pass preallocated
    pinned (S, dI, du0).  sync=True (default) waits for the device's current
    stream, so the returned tensors are complete, and raises LifbError if a
    kernel reported a device-side error; sync=False returns at once (the
    results are valid after the stream has drained)."""
    if I.is_cuda or GS.is_cuda:
        raise ValueError("lif_tuned_host takes host tensors; use lif_tuned for CUDA tensors")
    if I.dtype != torch.float32 or GS.dtype != torch.float32:
        raise TypeError("I and GS must be float32")
    I = I.contiguous()
    GS = GS.contiguous()
    T, N = I.shape
    if tuple(GS.shape) != (T, N):
        raise ValueError("GS must have the shape of I")
    u0 = torch.zeros(N, dtype=torch.float32) if u0 is None else u0.contiguous()
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    rows = block_n is None and N % 4 == 0
    if rows and block_t is not None and block_t <= 0:
        raise ValueError("block_t must be positive")
    if not rows and block_t is not None:
        raise ValueError("block_t applies to the row-block pipeline (N % 4 == 0, block_n not given)")
    if block_n is None and not rows:  # about 4 blocks, 128-neuron aligned
        block_n = max(128, ((N + 3) // 4 + 127) // 128 * 128)
    if out is None:
        out = (torch.empty(T, N).pin_memory(), torch.empty(T, N).pin_memory(), torch.empty(N).pin_memory())
    S, dI, du0 = out
    L = _lib.load()
    with torch.cuda.device(dev):
        st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        if rows:
            bt = int(block_t) if block_t is not None else L.lifb_lif_fwd_bwd_host_rows_block(T, N)
            nb = L.lifb_lif_fwd_bwd_host_rows_workspace_bytes(T, N, bt)
            ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)
            check(L.lifb_lif_fwd_bwd_host_rows(ptr(I), ptr(GS), ptr(u0), ptr(S), ptr(dI), ptr(du0), T, N,
                                               _f(beta), _f(theta), _f(u_r), _f(alpha), bt, ptr(ws), nb, st),
                  "lif_tuned_host")
        else:
            nb = L.lifb_lif_fwd_bwd_host_workspace_bytes(T, N, block_n)
            ws = torch.empty(max(nb, 1), dtype=torch.uint8, device=dev)
            check(L.lifb_lif_fwd_bwd_host(ptr(I), ptr(GS), ptr(u0), ptr(S), ptr(dI), ptr(du0), T, N, _f(beta),
                                          _f(theta), _f(u_r), _f(alpha), int(block_n), ptr(ws), nb, st),
                  "lif_tuned_host")
        if sync:
            # the host buffers are complete only once the stream has drained;
            # the device status is read at the same point
            torch.cuda.current_stream(dev).synchronize()
            _lib.check_device("lif_tuned_host")
    return S, dI, du0
