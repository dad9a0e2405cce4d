"""GPU forward parity through the C ABI: U and S bit-identical to the serial
fp32 recurrence (the CPU oracle, itself pinned to lifscan/fast.py), and the
scan's stats equal to the oracle's (hence the reference's).

Grids follow the reference's GPU tests: tests/test_triton.py:10-26 (beta x
drift x K, u_r = -0.1, u0 ~ N(0, 0.3^2)), tests/test_triton_tiled.py:6-20
(ragged widths), experiments/test_v3.py:12-22 and experiments/test_v4.py:6-20.
"""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_bit_equal, gen, to_dev

pytestmark = pytest.mark.gpu

BETAS = (0.5, 0.9, 0.99, 1.0)
DRIFTS = ((0.15, 0.4), (-0.1, 0.6), (0.4, 0.2))
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def L():
    from hard_resets_compose_b200 import lifscan
    return lifscan


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("N,T", ((100, 4096), (1000, 2048), (5000, 1024), (1, 300), (33, 7)))
def test_serial_forward_bit_exact(cuda, N, T):
    I, u0 = gen(T, N, 0.15, 0.4, seed=1, u0_sd=0.2)
    Us, Ss = O.serial_forward(I, 0.9, 1.0, -0.1, u0)
    Id, u0d = to_dev(cuda, I, u0)
    U, S = L().serial_forward(Id, 0.9, 1.0, -0.1, u0d)
    assert_bit_equal(_np(U), Us, "U")
    assert_bit_equal(_np(S), Ss, "S")


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "fwd_*.npz"))), ids=os.path.basename)
def test_golden_reference_outputs_and_stats(cuda, path):
    """Against the reference's own outputs (fast.py) and the stats of its v3
    kernels (stored by tests/golden/make_golden.py)."""
    z = np.load(path)
    beta, theta, u_r, C, K = (float(v) for v in z["params"])
    Id, u0d = to_dev(cuda, z["I"], z["u0"])
    U, S = L().serial_forward(Id, beta, theta, u_r, u0d)
    assert_bit_equal(_np(U), z["U"], "serial U")
    assert_bit_equal(_np(S), z["S"], "serial S")
    st = {}
    U, S = L().scan_forward_v3(Id, beta, theta, u_r, u0d, C=int(C), K=int(K), stats=st)
    assert_bit_equal(_np(U), z["U"], "v3 U")
    assert_bit_equal(_np(S), z["S"], "v3 S")
    ref = {str(k): float(v) for k, v in zip(z["stats_keys"], z["stats_vals"])}
    assert st["repair_iters"] == int(ref["repair_iters"])
    assert st["max_pieces"] == int(ref["max_pieces"])
    assert abs(st["overflow_frac"] - ref["overflow_frac"]) < 1e-6
    assert abs(st["mean_pieces"] - ref["mean_pieces"]) < 1e-5


@pytest.mark.parametrize("beta", BETAS)
@pytest.mark.parametrize("mu,sd", DRIFTS)
@pytest.mark.parametrize("K", (4, 16, 64))
def test_v3_bit_exact_and_stats(cuda, beta, mu, sd, K):
    T, N = 4096, 1000
    I, u0 = gen(T, N, mu, sd, seed=0, u0_sd=0.3)
    Us, Ss = O.serial_forward(I, beta, 1.0, -0.1, u0)
    _, _, ost = O.scan_forward_v3(I, beta, 1.0, -0.1, u0, C=64, K=K)
    Id, u0d = to_dev(cuda, I, u0)
    st = {}
    U, S = L().scan_forward_v3(Id, beta, 1.0, -0.1, u0d, C=64, K=K, stats=st)
    assert_bit_equal(_np(U), Us, "U")
    assert_bit_equal(_np(S), Ss, "S")
    assert st["repair_iters"] == ost["repair_iters"]
    assert st["max_pieces"] == ost["max_pieces"]
    assert abs(st["overflow_frac"] - ost["overflow_frac"]) < 1e-12
    assert abs(st["mean_pieces"] - ost["mean_pieces"]) < 1e-9


@pytest.mark.parametrize("beta", BETAS)
@pytest.mark.parametrize("mu,sd", DRIFTS)
@pytest.mark.parametrize("K,K2", ((16, 32), (8, 16)))
def test_v4_bit_exact_and_stats(cuda, beta, mu, sd, K, K2):
    T, N = 8192, 777
    I, u0 = gen(T, N, mu, sd, seed=0, u0_sd=0.3)
    Us, Ss = O.serial_forward(I, beta, 1.0, -0.1, u0)
    _, _, ost = O.scan_forward_v4(I, beta, 1.0, -0.1, u0, C=64, G=16, K=K, K2=K2)
    Id, u0d = to_dev(cuda, I, u0)
    st = {}
    U, S = L().scan_forward_v4(Id, beta, 1.0, -0.1, u0d, C=64, G=16, K=K, K2=K2, stats=st)
    assert_bit_equal(_np(U), Us, "U")
    assert_bit_equal(_np(S), Ss, "S")
    for k in ("repair_iters", "super_max_pieces"):
        assert st[k] == ost[k], k
    for k in ("overflow_frac", "super_overflow_frac", "mean_pieces", "super_mean_pieces"):
        assert abs(st[k] - ost[k]) < 1e-9, k


@pytest.mark.parametrize("C,K", ((8, 1), (16, 2), (32, 4), (256, 8), (1024, 16)))
def test_v3_chunk_shapes_and_overflow(cuda, C, K):
    """Tiny capacities force the in-carry serial fallback; C = T is one chunk."""
    T, N = 1024, 257
    I, u0 = gen(T, N, 0.2, 0.5, seed=7, u0_sd=0.3)
    Us, Ss = O.serial_forward(I, 0.95, 1.0, 0.0, u0)
    Id, u0d = to_dev(cuda, I, u0)
    st = {}
    U, S = L().scan_forward_v3(Id, 0.95, 1.0, 0.0, u0d, C=C, K=K, stats=st)
    assert_bit_equal(_np(U), Us, "U")
    assert_bit_equal(_np(S), Ss, "S")
    _, _, ost = O.scan_forward_v3(I, 0.95, 1.0, 0.0, u0, C=C, K=K)
    assert st["overflow_frac"] == pytest.approx(ost["overflow_frac"], abs=1e-12)


def test_c1_full_size_bit_exact(cuda):
    """Config 1: B*N = 4096, T = 1024, x ~ N(0.1, 0.3^2), beta = 0.9."""
    I, u0 = gen(1024, 4096, 0.1, 0.3, seed=0)
    Us, Ss = O.serial_forward(I, 0.9, 1.0, 0.0, u0)
    Id, u0d = to_dev(cuda, I, u0)
    for fn in (lambda: L().scan_forward_auto(Id, 0.9, 1.0, 0.0, u0d),
               lambda: L().scan_forward_v3(Id, 0.9, 1.0, 0.0, u0d, C=64, K=16),
               lambda: L().serial_forward_auto(Id, 0.9, 1.0, 0.0, u0d)):
        U, S = fn()
        assert_bit_equal(_np(U), Us, "U")
        assert_bit_equal(_np(S), Ss, "S")


def test_c2_full_size_bit_exact(cuda):
    """Config 2 forward: B*N = 16384, T = 1024, x ~ N(0.05, 0.2^2), beta = 0.99."""
    I, u0 = gen(1024, 16384, 0.05, 0.2, seed=0)
    Us, Ss = O.serial_forward(I, 0.99, 1.0, 0.0, u0)
    Id, u0d = to_dev(cuda, I, u0)
    U, S = L().scan_forward_auto(Id, 0.99, 1.0, 0.0, u0d)
    assert_bit_equal(_np(U), Us, "U")
    assert_bit_equal(_np(S), Ss, "S")


def test_long_sequence_v4_properties(cuda):
    """Long-T three-level path at reduced T (T = 2^18, B*N = 1024): exact
    against the oracle's serial recurrence."""
    T, N = 1 << 18, 1024
    I, u0 = gen(T, N, 0.02, 0.1, seed=0)
    Us, Ss = O.serial_forward(I, 0.99, 1.0, 0.0, u0)
    Id, u0d = to_dev(cuda, I, u0)
    U, S = L().scan_forward_v4(Id, 0.99, 1.0, 0.0, u0d, C=64, G=16, K=16, K2=32)
    assert_bit_equal(_np(S), Ss, "S")
    assert_bit_equal(_np(U), Us, "U")


def test_empty_inputs(cuda):
    I = torch.empty(0, 5, device=cuda)
    U, S = L().serial_forward(I, 0.9, 1.0, 0.0, torch.zeros(5, device=cuda))
    assert U.shape == (0, 5)
    I = torch.empty(64, 0, device=cuda)
    U, S = L().scan_forward_v3(I, 0.9, 1.0, 0.0, torch.zeros(0, device=cuda))
    assert U.shape == (64, 0)


def test_bad_arguments_raise(cuda):
    I = torch.zeros(100, 4, device=cuda)
    with pytest.raises(ValueError):
        L().scan_forward_v3(I, 0.9, 1.0, 0.0, torch.zeros(4, device=cuda), C=64)
    with pytest.raises(Exception):
        L().scan_forward_v3(torch.zeros(128, 4, device=cuda), 0.9, 1.0, 0.0, torch.zeros(4, device=cuda), C=64,
                            K=65)
    with pytest.raises(ValueError):
        L().serial_forward(I, 0.9, 1.0, 0.0, torch.zeros(5, device=cuda))


@pytest.mark.parametrize("beta", BETAS)
@pytest.mark.parametrize("mu,sd", DRIFTS)
@pytest.mark.parametrize("N", (1000, 777))
def test_v3_fast_path_bit_exact(cuda, beta, mu, sd, N):
    """Without stats the v3 forward replays long segments from the carried
    starts and fixes the inexact ones (N = 1000: TMA kernels; N = 777: the
    N % 4 != 0 fallback)."""
    T = 4096
    I, u0 = gen(T, N, mu, sd, seed=11, u0_sd=0.3)
    Us, Ss = O.serial_forward(I, beta, 1.0, -0.1, u0)
    Id, u0d = to_dev(cuda, I, u0)
    for K in (4, 16):
        U, S = L().scan_forward_v3(Id, beta, 1.0, -0.1, u0d, C=64, K=K)
        assert_bit_equal(_np(U), Us, f"U K={K}")
        assert_bit_equal(_np(S), Ss, f"S K={K}")


@pytest.mark.parametrize("beta", BETAS)
@pytest.mark.parametrize("mu,sd", DRIFTS)
def test_v4_fast_path_bit_exact(cuda, beta, mu, sd):
    T, N = 8192, 1000
    I, u0 = gen(T, N, mu, sd, seed=12, u0_sd=0.3)
    Us, Ss = O.serial_forward(I, beta, 1.0, -0.1, u0)
    Id, u0d = to_dev(cuda, I, u0)
    for (C, G, K, K2) in ((64, 16, 16, 32), (32, 8, 4, 8)):
        U, S = L().scan_forward_v4(Id, beta, 1.0, -0.1, u0d, C=C, G=G, K=K, K2=K2)
        assert_bit_equal(_np(U), Us, f"U {C},{G},{K},{K2}")
        assert_bit_equal(_np(S), Ss, f"S {C},{G},{K},{K2}")


def test_long_sequence_v3_fast_path(cuda):
    """Two-level path at long T (T = 2^17, B*N = 1024): the staged carry runs
    2048 maps per neuron; config 4's input distribution."""
    T, N = 1 << 17, 1024
    I, u0 = gen(T, N, 0.02, 0.1, seed=0)
    Us, Ss = O.serial_forward(I, 0.99, 1.0, 0.0, u0)
    Id, u0d = to_dev(cuda, I, u0)
    U, S = L().scan_forward_v3(Id, 0.99, 1.0, 0.0, u0d, C=64, K=16)
    assert_bit_equal(_np(S), Ss, "S")
    assert_bit_equal(_np(U), Us, "U")


@pytest.mark.parametrize("beta,mu,sd", ((0.99, 0.02, 0.1), (0.9, 0.15, 0.4), (1.0, -0.01, 0.05), (0.5, 0.4, 0.2)))
@pytest.mark.parametrize("N,T,Lseg,W", ((1024, 1 << 16, 4096, 1024), (1000, 1 << 15, 2048, 0), (64, 1 << 15, 1024, 4096),
                                     (2048, 8192, 512, 256), (777, 1 << 14, 1024, 1024)))
def test_spec_forward_bit_exact(cuda, beta, mu, sd, N, T, Lseg, W):
    """Speculative segment forward: W-row lead-ins (W = 0: every guess is u_r,
    W > L: lead-ins span several segments), N % 4 != 0 on the plain replay."""
    I, u0 = gen(T, N, mu, sd, seed=21, u0_sd=0.3)
    Us, Ss = O.serial_forward(I, beta, 1.0, -0.1, u0)
    Id, u0d = to_dev(cuda, I, u0)
    U, S = L().scan_forward_spec(Id, beta, 1.0, -0.1, u0d, L=Lseg, W=W)
    assert_bit_equal(_np(U), Us, "U")
    assert_bit_equal(_np(S), Ss, "S")


def test_spec_forward_c4_reduced_auto(cuda):
    """The auto policy at config 4's width and distribution (T = 2^18)."""
    T, N = 1 << 18, 1024
    I, u0 = gen(T, N, 0.02, 0.1, seed=0)
    Us, Ss = O.serial_forward(I, 0.99, 1.0, 0.0, u0)
    Id, u0d = to_dev(cuda, I, u0)
    assert L().spec_segment(T, N)[0] < T
    U, S = L().scan_forward_auto(Id, 0.99, 1.0, 0.0, u0d)
    assert_bit_equal(_np(S), Ss, "S")
    assert_bit_equal(_np(U), Us, "U")


@pytest.mark.parametrize("N,T,W", ((1024, 1 << 15, 4096), (1000, 8192, 512)))
def test_spec_forward_halo(cuda, N, T, W):
    """With a halo (the rows before row 0) and u0 the guess before it, the
    result is the recurrence from the state the halo leads to."""
    I, _ = gen(T + W, N, 0.02, 0.1, seed=5)
    guess = np.zeros(N, np.float32)
    Uh, _ = O.serial_forward(I[:W], 0.99, 1.0, 0.0, guess)
    Us, Ss = O.serial_forward(I[W:], 0.99, 1.0, 0.0, Uh[-1].copy())
    Id, gd = to_dev(cuda, I, guess)
    U, S = L().scan_forward_spec(Id[W:], 0.99, 1.0, 0.0, gd, halo=Id[:W])
    assert_bit_equal(_np(S), Ss, "S")
    assert_bit_equal(_np(U), Us, "U")


def test_spec_begin_finish(cuda):
    """The two-call form: _finish alone is exact for its u0; the end guess is
    the last W rows run from u_r."""
    from hard_resets_compose_b200 import _lib
    T, N, Lseg, W = 1 << 16, 1024, 16384, 4096
    I, u0 = gen(T, N, 0.02, 0.1, seed=9, u0_sd=0.3)
    Us, Ss = O.serial_forward(I, 0.99, 1.0, 0.0, u0)
    Ug, _ = O.serial_forward(I[-W:], 0.99, 1.0, 0.0, np.zeros(N, np.float32))
    Id, u0d = to_dev(cuda, I, u0)
    lib = _lib.load()
    nb = lib.lifb_scan_fwd_spec_workspace_bytes(T, N, Lseg)
    ws = torch.empty(nb, dtype=torch.uint8, device=cuda)
    g = torch.empty(N, device=cuda)
    U = torch.empty_like(Id)
    S = torch.empty_like(Id)
    st = _lib.stream_of(Id)
    _lib.check(lib.lifb_scan_fwd_spec_begin(_lib.ptr(Id), T, N, 0.99, 1.0, 0.0, Lseg, W, _lib.ptr(g), _lib.ptr(ws), nb,
                                            st), "begin")
    _lib.check(lib.lifb_scan_fwd_spec_finish(_lib.ptr(Id), _lib.ptr(u0d), _lib.ptr(U), _lib.ptr(S), T, N, 0.99, 1.0,
                                             0.0, Lseg, _lib.ptr(ws), nb, st), "finish")
    assert_bit_equal(_np(U), Us, "U")
    assert_bit_equal(_np(S), Ss, "S")
    assert_bit_equal(_np(g), Ug[-1], "end guess")
