"""ctypes wrapper of the CPU oracle (oracle/lif_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()`` and
by bench.py's CPU-baseline / ``--impl reference`` legs, always as the checker or
the timed CPU baseline, never as the product path.  The product package
``hard_resets_compose_b200`` never imports this module.

Every function takes and returns numpy float32 arrays in the reference layout
([T, N] row-major, neuron index fastest) and follows the reference function it
names (file:line in lifscan/):
  serial_forward       fast.py:69-81
  serial_backward      fast.py:227-239
  envelope             triton_lif.py:698-733
  build_maps           triton_lif.py:736-779   (spec fast.py:147-183)
  carry                triton_lif.py:578-606   (spec fast.py:242-251)
  scan_forward_v3      triton_lif.py:782-817
  scan_forward_v4      triton_lif.py:935-983
  scan_backward        triton_lif.py:512-526
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

f32p = ctypes.POINTER(ctypes.c_float)
i32p = ctypes.POINTER(ctypes.c_int32)
f64p = ctypes.POINTER(ctypes.c_double)
i64 = ctypes.c_int64
c_float = ctypes.c_float
c_int = ctypes.c_int


class OracleStats(ctypes.Structure):
    _fields_ = [
        ("repair_iters", ctypes.c_int),
        ("max_pieces", ctypes.c_int),
        ("super_max_pieces", ctypes.c_int),
        ("_pad", ctypes.c_int),
        ("overflow_frac", ctypes.c_double),
        ("mean_pieces", ctypes.c_double),
        ("super_overflow_frac", ctypes.c_double),
        ("super_mean_pieces", ctypes.c_double),
    ]


def build() -> str:
    """Compile liboracle.so with the Makefile beside this file."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "lif_oracle.c"))
        ):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        L.oracle_serial_fwd.argtypes = [f32p, f32p, f32p, f32p, f32p, i64, i64, c_float, c_float, c_float]
        L.oracle_soft_serial_fwd.argtypes = [f32p, f32p, f32p, f32p, f32p, i64, i64, c_float, c_float]
        L.oracle_soft_serial_bwd.argtypes = [f32p, f32p, f32p, f32p, f32p, i64, i64, c_float, c_float, c_float,
                                             c_int]
        L.oracle_alif_serial_fwd.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, i64, i64, c_float, c_float,
                                             c_float, c_float, c_float]
        L.oracle_alif_serial_bwd.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, f32p, f64p,
                                             i64, i64, c_float, c_float, c_float, c_float, c_float, c_int]
        L.oracle_aff_serial_fwd.argtypes = [f32p, f32p, f32p, f32p, f32p, i64, i64, c_float, c_float, c_float,
                                            c_float]
        L.oracle_aff_serial_bwd.argtypes = [f32p, f32p, f32p, f32p, f32p, f64p, i64, i64, c_float, c_float,
                                            c_float, c_float, c_int]
        L.oracle_serial_bwd.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, f32p, i64, i64,
                                        c_float, c_float, c_float, c_float, c_int]
        L.oracle_envelope.argtypes = [f32p, f32p, f32p, i64, i64, c_int, c_float, c_float, c_float]
        L.oracle_build_maps.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, f32p, i32p, i32p,
                                        i64, i64, c_int, c_int, c_float, c_float, c_float]
        L.oracle_carry.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, i32p, i32p, f32p,
                                   i64, i64, i64, c_int, c_float, c_float, c_float]
        L.oracle_replay_repair.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, i64, i64, c_int,
                                           c_float, c_float, c_float, c_int]
        L.oracle_replay_repair.restype = c_int
        L.oracle_scan_fwd_v3.argtypes = [f32p, f32p, f32p, f32p, i64, i64, c_float, c_float, c_float,
                                         c_int, c_int, c_int,
                                         f32p, f32p, f32p, f32p, f32p, i32p, i32p, f32p, f32p,
                                         ctypes.POINTER(OracleStats)]
        L.oracle_scan_fwd_v4.argtypes = [f32p, f32p, f32p, f32p, i64, i64, c_float, c_float, c_float,
                                         c_int, c_int, c_int, c_int, c_int,
                                         f32p, f32p, f32p, f32p, f32p, i32p, i32p,
                                         f32p, f32p, f32p, f32p, i32p, i32p,
                                         f32p, f32p, f32p, ctypes.POINTER(OracleStats)]
        L.oracle_scan_bwd.argtypes = [f32p, f32p, f32p, f32p, f32p, f32p, f32p, i64, i64, c_int,
                                      c_float, c_float, c_float, c_float, c_int]
        L.oracle_num_threads.restype = c_int
        L.oracle_set_threads.argtypes = [c_int]
        _lib = L
    return _lib


def _f(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a


def _p(a):
    if a is None:
        return None
    if a.dtype == np.int32:
        return a.ctypes.data_as(i32p)
    return a.ctypes.data_as(f32p)


def num_threads() -> int:
    return lib().oracle_num_threads()


def set_threads(n: int) -> None:
    lib().oracle_set_threads(int(n))


def serial_forward(I, beta, theta, u_r, u0, want_v=False):
    I = _f(I)
    u0 = _f(u0)
    T, N = I.shape
    U = np.empty_like(I)
    S = np.empty_like(I)
    V = np.empty_like(I) if want_v else None
    lib().oracle_serial_fwd(_p(I), _p(u0), _p(U), _p(S), _p(V), T, N, beta, theta, u_r)
    return (U, S, V) if want_v else (U, S)


def serial_backward(I, u0, U, S, GS, GU, beta, theta, u_r, alpha=4.0, detach=True):
    I, u0, U, S, GS = map(_f, (I, u0, U, S, GS))
    GU = None if GU is None else _f(GU)
    T, N = I.shape
    Lam = np.empty_like(I)
    lib().oracle_serial_bwd(_p(I), _p(u0), _p(U), _p(S), _p(GS), _p(GU), _p(Lam), T, N,
                            beta, theta, u_r, alpha, int(bool(detach)))
    return Lam


def soft_serial_forward(I, beta, theta, u0, want_v=False):
    """Soft-reset recurrence (lifscan/triton_lif.py:1037-1049) -> (U, S[, V])."""
    I, u0 = _f(I), _f(u0)
    T, N = I.shape
    U = np.empty_like(I)
    S = np.empty_like(I)
    V = np.empty_like(I) if want_v else None
    lib().oracle_soft_serial_fwd(_p(I), _p(u0), _p(U), _p(S), _p(V), T, N, beta, theta)
    return (U, S, V) if want_v else (U, S)


def soft_serial_backward(I, u0, U, GS, beta, theta, alpha=4.0, double=False):
    """Soft-reset detached adjoint (lifscan/triton_lif.py:1052-1069), fp32 in the
    kernel's order, or in double (double=True)."""
    I, u0, U, GS = map(_f, (I, u0, U, GS))
    T, N = I.shape
    Lam = np.empty_like(I)
    lib().oracle_soft_serial_bwd(_p(I), _p(u0), _p(U), _p(GS), _p(Lam), T, N, beta, theta, alpha, int(double))
    return Lam


def aff_serial_forward(I, beta, theta, gamma, delta, u0, want_v=False):
    """Affine-reset recurrence (lifscan/triton_affine.py:19-23, 158-162) -> (U, S[, V])."""
    I, u0 = _f(I), _f(u0)
    T, N = I.shape
    U = np.empty_like(I)
    S = np.empty_like(I)
    V = np.empty_like(I) if want_v else None
    lib().oracle_aff_serial_fwd(_p(I), _p(u0), _p(U), _p(S), _p(V), T, N, beta, theta, gamma, delta)
    return (U, S, V) if want_v else (U, S)


def aff_serial_backward(I, u0, U, GS, beta, theta, gamma, alpha=4.0, double=False):
    """Affine-reset detached adjoint and (dbeta, dgamma, ddelta)
    (lifscan/triton_affine.py:229-238) -> (Lam, pg), fp32 in order or in
    double (double=True)."""
    I, u0, U, GS = map(_f, (I, u0, U, GS))
    T, N = I.shape
    Lam = np.empty_like(I)
    pg = np.zeros(3, np.float64)
    lib().oracle_aff_serial_bwd(_p(I), _p(u0), _p(U), _p(GS), _p(Lam), pg.ctypes.data_as(f64p), T, N, beta, theta, alpha, gamma, int(double))
    return Lam, pg


def alif_serial_forward(I, beta, rho, q, theta0, u_r, u0, w0):
    """ALIF recurrence (lifscan/triton_alif.py:25-42, 263-273) -> (U, W, S)."""
    I, u0, w0 = _f(I), _f(u0), _f(w0)
    T, N = I.shape
    U = np.empty_like(I)
    W = np.empty_like(I)
    S = np.empty_like(I)
    lib().oracle_alif_serial_fwd(_p(I), _p(u0), _p(w0), _p(U), _p(W), _p(S), T, N, beta, rho, q, theta0, u_r)
    return U, W, S


def alif_serial_backward(I, u0, w0, U, W, S, GS, beta, rho, q, theta0, alpha=4.0, double=False):
    """ALIF detached adjoint (lifscan/triton_alif.py:366-431, PASS 4) and the
    ALIFFn parameter gradients (:542-554) -> (LV, LW, lw_m1, pg) with pg =
    (dbeta, drho, dq, dtheta0); fp32 in the kernel's order, or in double."""
    I, u0, w0, U, W, S, GS = map(_f, (I, u0, w0, U, W, S, GS))
    T, N = I.shape
    LV = np.empty_like(I)
    LW = np.empty_like(I)
    lwm1 = np.empty(N, np.float32)
    pg = np.zeros(4, np.float64)
    lib().oracle_alif_serial_bwd(_p(I), _p(u0), _p(w0), _p(U), _p(W), _p(S), _p(GS), _p(LV), _p(LW), _p(lwm1),
                                 pg.ctypes.data_as(f64p), T, N, beta, rho, q, theta0, alpha, int(double))
    return LV, LW, lwm1, pg


def alif_warm_predict(I, beta, rho, q, theta0, u_r, u0, w0, C, Wn=4, u_init=0.0, w_init=0.0, UI=None, WI=None):
    """lifscan/triton_alif.py:74-92: WP[m] = w after the Wn chunks before chunk
    m, from (u_init, w_init) or (UI, WI)[m - Wn], or (u0, w0) from row 0."""
    I, u0, w0 = _f(I), _f(u0), _f(w0)
    T, N = I.shape
    M = T // C
    WP = np.empty((M, N), np.float32)
    for m in range(M):
        s0 = max(m - Wn, 0)
        if s0 == 0:
            u, w = u0, w0
        elif UI is not None:
            u, w = _f(UI)[s0], _f(WI)[s0]
        else:
            u = np.full(N, u_init, np.float32)
            w = np.full(N, w_init, np.float32)
        if m * C > s0 * C:
            Us, Ws, _ = alif_serial_forward(I[s0 * C:m * C], beta, rho, q, theta0, u_r, u, w)
            w = Ws[-1]
        WP[m] = w
    return WP


def envelope(I, u0, C, beta, u_r, margin=1e-5):
    I = _f(I)
    u0 = _f(u0)
    T, N = I.shape
    Lo = np.empty((T // C, N), np.float32)
    lib().oracle_envelope(_p(I), _p(u0), _p(Lo), T, N, C, beta, u_r, margin)
    return Lo


def _maps(M, N, K):
    return dict(
        MA=np.empty((M, N), np.float32), MB=np.empty((M, N), np.float32),
        MX=np.empty((M, K, N), np.float32), MC=np.empty((M, K, N), np.float32),
        MN=np.empty((M, N), np.int32), OVF=np.empty((M, N), np.int32),
    )


def build_maps(I, u0, Lo, C, K, beta, theta, u_r):
    I, u0, Lo = _f(I), _f(u0), _f(Lo)
    T, N = I.shape
    d = _maps(T // C, N, K)
    lib().oracle_build_maps(_p(I), _p(u0), _p(Lo), _p(d["MA"]), _p(d["MB"]), _p(d["MX"]), _p(d["MC"]),
                            _p(d["MN"]), _p(d["OVF"]), T, N, C, K, beta, theta, u_r)
    return d


def scan_forward_v3(I, beta, theta, u_r, u0, C=64, K=16, repair=10 ** 6, return_internals=False):
    """Returns (U, S, stats[, internals])."""
    I, u0 = _f(I), _f(u0)
    T, N = I.shape
    if T % C:
        raise ValueError("T must be a multiple of C")
    M = T // C
    d = _maps(M, N, K)
    d["Lo"] = np.empty((M, N), np.float32)
    d["Starts"] = np.empty((M, N), np.float32)
    d["Ends"] = np.empty((M, N), np.float32)
    U = np.empty_like(I)
    S = np.empty_like(I)
    st = OracleStats()
    lib().oracle_scan_fwd_v3(_p(I), _p(u0), _p(U), _p(S), T, N, beta, theta, u_r, C, K, int(repair),
                             _p(d["Lo"]), _p(d["MA"]), _p(d["MB"]), _p(d["MX"]), _p(d["MC"]),
                             _p(d["MN"]), _p(d["OVF"]), _p(d["Starts"]), _p(d["Ends"]), ctypes.byref(st))
    stats = dict(repair_iters=st.repair_iters, overflow_frac=st.overflow_frac,
                 mean_pieces=st.mean_pieces, max_pieces=st.max_pieces)
    if return_internals:
        return U, S, stats, d
    return U, S, stats


def scan_forward_v4(I, beta, theta, u_r, u0, C=64, G=16, K=16, K2=32, repair=10 ** 6,
                    return_internals=False):
    I, u0 = _f(I), _f(u0)
    T, N = I.shape
    M = T // C
    if T % C or M % G:
        raise ValueError("T must be divisible by C*G")
    M2 = M // G
    d = _maps(M, N, K)
    d["Lo"] = np.empty((M, N), np.float32)
    d["Starts"] = np.empty((M, N), np.float32)
    d["Ends"] = np.empty((M, N), np.float32)
    d.update(SA=np.empty((M2, N), np.float32), SB=np.empty((M2, N), np.float32),
             SX=np.empty((M2, K2, N), np.float32), SC=np.empty((M2, K2, N), np.float32),
             SN=np.empty((M2, N), np.int32), SOVF=np.empty((M2, N), np.int32),
             SStarts=np.empty((M2, N), np.float32))
    U = np.empty_like(I)
    S = np.empty_like(I)
    st = OracleStats()
    lib().oracle_scan_fwd_v4(_p(I), _p(u0), _p(U), _p(S), T, N, beta, theta, u_r, C, G, K, K2, int(repair),
                             _p(d["Lo"]), _p(d["MA"]), _p(d["MB"]), _p(d["MX"]), _p(d["MC"]),
                             _p(d["MN"]), _p(d["OVF"]),
                             _p(d["SA"]), _p(d["SB"]), _p(d["SX"]), _p(d["SC"]), _p(d["SN"]), _p(d["SOVF"]),
                             _p(d["SStarts"]), _p(d["Starts"]), _p(d["Ends"]), ctypes.byref(st))
    stats = dict(repair_iters=st.repair_iters, overflow_frac=st.overflow_frac,
                 super_overflow_frac=st.super_overflow_frac, mean_pieces=st.mean_pieces,
                 super_mean_pieces=st.super_mean_pieces, super_max_pieces=st.super_max_pieces)
    if return_internals:
        return U, S, stats, d
    return U, S, stats


def scan_backward(I, u0, U, S, GS, GU, beta, theta, u_r, alpha=4.0, detach=True, C=64):
    I, u0, U, S, GS = map(_f, (I, u0, U, S, GS))
    GU = None if GU is None else _f(GU)
    T, N = I.shape
    if T % C:
        raise ValueError("T must be a multiple of C")
    Lam = np.empty_like(I)
    lib().oracle_scan_bwd(_p(I), _p(u0), _p(U), _p(S), _p(GS), _p(GU), _p(Lam), T, N, C,
                          beta, theta, u_r, alpha, int(bool(detach)))
    return Lam


def gen_inputs(T, N, mu, sd, seed=0, u0_sd=0.0, grad=False):
    """Seeded inputs, generated on the CPU with torch.Generator exactly as the
    reference's tests do (tests/test_fast.py:7-9): I = mu + sd*randn(T, N);
    u0 = u0_sd*randn(N) (zeros when u0_sd == 0); GS = randn(T, N)."""
    import torch
    g = torch.Generator().manual_seed(seed)
    I = (mu + sd * torch.randn(T, N, generator=g)).to(torch.float32)
    if u0_sd:
        u0 = (u0_sd * torch.randn(N, generator=g)).to(torch.float32)
    else:
        u0 = torch.zeros(N, dtype=torch.float32)
    GS = torch.randn(T, N, generator=g).to(torch.float32) if grad else None
    out = (I.numpy(), u0.numpy())
    return out + (GS.numpy(),) if grad else out
