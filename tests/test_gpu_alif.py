"""Adaptive-threshold LIF (ALIF) on the GPU through the C ABI: U, W, S
bit-identical to the reference's serial recurrence and exact box scan (stored
outputs over the neuron classes of its tests/test_alif.py,
tests/golden/alif_grid.npz, and the oracle those pin) for any prediction of
the entry adaptation; warm-up predictions bit for bit; the adjoint pair and
ALIFFn's gradients for I, u0, w0, beta, rho, q, theta0 within 1e-5
(lifscan/triton_alif.py)."""
import math
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_bit_equal, rel, to_dev

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "alif_grid.npz")
TOL = 1e-5
KEYS = [f"a{c}m{m}" for c in range(3) for m in range(2)]
CLASSES = (("lsnn", 0.95, 0.995, 0.9), ("glif2", 0.99, 0.96, 0.2), ("appD-a", 0.9, 0.95, 0.5))


def _np(t):
    return t.detach().cpu().numpy()


def _param_close(got, want, scale=0.0):
    """A parameter gradient is a sum over T*N neuron-steps that can cancel to
    far below its summands (drho: |sum| / sum|terms| ~ 1e-5 at config 2's
    width), so it is held to 1e-5 of itself plus 1e-6 of sum|terms|: the sum
    agrees as well as its summands do."""
    return abs(got - want) <= TOL * (abs(want) + 1e-3) + 1e-6 * scale


def _scales(I, u0, w0, U, W, S, GS, LV, LW, beta, q, theta0, alpha=4.0):
    """sum|terms| of (dbeta, drho, dq, dtheta0) (lifscan/triton_alif.py:546-553)."""
    Up = np.concatenate([u0[None], U[:-1]], 0).astype(np.float64)
    Wp = np.concatenate([w0[None], W[:-1]], 0).astype(np.float64)
    v = beta * Up + I
    sig = 1.0 / (1.0 + np.exp(-alpha * (v - theta0 - Wp)))
    sg = alpha * sig * (1.0 - sig)
    d = GS + q * LW.astype(np.float64)
    return (np.abs(LV * Up).sum(), np.abs(LW * Wp).sum(), np.abs(LW * S).sum(), np.abs(sg * d).sum())


def _gen(T, N, beta, mfree, seed, grad=False):
    """Inputs as the reference's tests draw them (tests/test_alif.py:13-16)."""
    rng = np.random.default_rng(seed)
    I = ((1 - beta) * mfree + 0.5 * math.sqrt(1 - beta * beta) * rng.standard_normal((T, N))).astype(np.float32)
    u0 = np.zeros(N, np.float32)
    w0 = (0.1 * rng.random(N)).astype(np.float32)
    if grad:
        return I, u0, w0, rng.standard_normal((T, N)).astype(np.float32)
    return I, u0, w0


@pytest.mark.parametrize("key", KEYS)
def test_alif_golden(cuda, key):
    from hard_resets_compose_b200 import alif as A
    z = np.load(GOLD)
    beta, rho, q, theta0, u_r, alpha = (float(v) for v in z[f"{key}_params"])
    Id, u0d, w0d, GSd, WPd = to_dev(cuda, *(z[f"{key}_{k}"] for k in ("I", "u0", "w0", "GS", "WP")))
    WP = A.alif_warm_predict(Id, beta, rho, q, theta0, u_r, u0d, w0d, 32, Wn=4)
    assert_bit_equal(_np(WP), z[f"{key}_WP"], "WP")
    for U, W, S in (A.alif_serial_forward(Id, beta, rho, q, theta0, u_r, u0d, w0d),
                    A.alif_serial_forward(Id, beta, rho, q, theta0, u_r, u0d, w0d, D=8),
                    A.alif_scan_forward(Id, beta, rho, q, theta0, u_r, u0d, w0d, WPd, 0.1 * q, C=32,
                                        repair=10 ** 6)):
        assert_bit_equal(_np(U), z[f"{key}_U"], "U")
        assert_bit_equal(_np(W), z[f"{key}_W"], "W")
        assert_bit_equal(_np(S), z[f"{key}_S"], "S")
    Ud, Wd, Sd = to_dev(cuda, z[f"{key}_U"], z[f"{key}_W"], z[f"{key}_S"])
    for mode in ("serial", "scan"):
        LV, LW = A.alif_backward(Id, Ud, Wd, Sd, GSd, beta, rho, q, theta0, u0d, w0d, alpha=alpha, mode=mode, C=32)
        assert rel(_np(LV), z[f"{key}_LV"]) < TOL
        assert rel(_np(LW), z[f"{key}_LW"]) < TOL
    dp = z[f"{key}_dp"].astype(np.float64)
    sc = _scales(*(z[f"{key}_{k}"] for k in ("I", "u0", "w0", "U", "W", "S", "GS", "LV", "LW")), beta, q, theta0,
                 alpha)
    Ig = Id.clone().requires_grad_(True)
    ug = u0d.clone().requires_grad_(True)
    wg = w0d.clone().requires_grad_(True)
    ps = [torch.tensor(v, device=cuda, requires_grad=True) for v in (beta, rho, q, theta0)]
    S, _, _ = A.alif(Ig, ug, wg, ps[0], ps[1], ps[2], ps[3], u_r=u_r, alpha=alpha, fwd="serial", bwd="serial")
    torch.autograd.backward(S, GSd)
    assert_bit_equal(_np(S), z[f"{key}_S"], "S")
    assert rel(_np(Ig.grad), z[f"{key}_dI"]) < TOL
    assert rel(_np(ug.grad), z[f"{key}_du0"]) < TOL
    assert rel(_np(wg.grad), z[f"{key}_dw0"]) < TOL
    for i in range(4):
        assert _param_close(float(ps[i].grad), dp[i], sc[i]), (i, float(ps[i].grad), dp[i])


@pytest.mark.parametrize("mfree", (0.5, 2.0))
@pytest.mark.parametrize("cls", CLASSES, ids=lambda c: c[0])
@pytest.mark.parametrize("pred", ("none", "warm", "bad"))
def test_alif_scan_bit_exact(cuda, cls, mfree, pred):
    """The speculative ALIF scan where segments and lead-ins apply, for no
    prediction, the warm-up prediction and a deliberately wrong one (every
    entry adaptation off by 5q, tests/test_alif.py:25)."""
    from hard_resets_compose_b200 import alif as A
    _, beta, rho, q = cls
    T, N, C = 1 << 16, 1024, 128
    I, u0, w0 = _gen(T, N, beta, mfree, seed=3)
    Us, Ws, Ss = O.alif_serial_forward(I, beta, rho, q, 1.0, 0.0, u0, w0)
    Id, u0d, w0d = to_dev(cuda, I, u0, w0)
    Wp = None
    if pred == "warm":
        Wp = A.alif_warm_predict(Id, beta, rho, q, 1.0, 0.0, u0d, w0d, C, Wn=4)
    elif pred == "bad":
        Wentry = np.concatenate([w0[None], Ws[C - 1:-1:C]], 0) + 5 * q
        Wp = to_dev(cuda, Wentry.astype(np.float32))[0]
    st = {}
    U, W, S = A.alif_scan_forward(Id, beta, rho, q, 1.0, 0.0, u0d, w0d, Wp, 0.1 * q, C=C, stats=st)
    assert st["segments"] > 1
    assert_bit_equal(_np(S), Ss, "S")
    assert_bit_equal(_np(W), Ws, "W")
    assert_bit_equal(_np(U), Us, "U")


@pytest.mark.parametrize("T,N,beta,rho,q", ((1 << 15, 256, 0.95, 1.0, 0.9), (8192, 333, 0.95, 0.995, 0.9),
                                            (1000, 77, 0.9, 0.95, 0.5), (1 << 14, 1000, 0.99, 0.96, 0.2)))
def test_alif_forward_hard_cases(cuda, T, N, beta, rho, q):
    """rho = 1 (the adaptation never forgets: a wrong guess never rejoins and
    the fix-up carries every segment), N % 4 != 0 (the plain kernels), T not a
    multiple of the tile."""
    from hard_resets_compose_b200 import alif as A
    I, u0, w0 = _gen(T, N, beta, 2.0, seed=5)
    Us, Ws, Ss = O.alif_serial_forward(I, beta, rho, q, 1.0, 0.0, u0, w0)
    Id, u0d, w0d = to_dev(cuda, I, u0, w0)
    for U, W, S in (A.alif_serial_forward(Id, beta, rho, q, 1.0, 0.0, u0d, w0d),
                    A.alif_scan_forward(Id, beta, rho, q, 1.0, 0.0, u0d, w0d, None, 0.1, C=T // 8 if T % 8 == 0
                                        else T, D=1)):
        assert_bit_equal(_np(S), Ss, "S")
        assert_bit_equal(_np(W), Ws, "W")
        assert_bit_equal(_np(U), Us, "U")


@pytest.mark.parametrize("T,N", ((4096, 8), (1024, 16384), (3000, 333), (1 << 15, 512), (1 << 14, 100)))
@pytest.mark.parametrize("cls", CLASSES, ids=lambda c: c[0])
def test_alif_backward(cuda, T, N, cls):
    """The adjoint pair (reading S, and with S recomputed) and the fused
    parameter sums against the oracle (the sums against its fp64 sweep)."""
    from hard_resets_compose_b200 import alif as A
    _, beta, rho, q = cls
    I, u0, w0, GS = _gen(T, N, beta, 2.0, seed=7, grad=True)
    U, W, S = O.alif_serial_forward(I, beta, rho, q, 1.0, 0.0, u0, w0)
    LV, LW, lwm1, _ = O.alif_serial_backward(I, u0, w0, U, W, S, GS, beta, rho, q, 1.0, 4.0)
    _, _, _, pg = O.alif_serial_backward(I, u0, w0, U, W, S, GS, beta, rho, q, 1.0, 4.0, double=True)
    sc = _scales(I, u0, w0, U, W, S, GS, LV, LW, beta, q, 1.0)
    Id, u0d, w0d, Ud, Wd, Sd, GSd = to_dev(cuda, I, u0, w0, U, W, S, GS)
    LVg, LWg = A.alif_backward(Id, Ud, Wd, Sd, GSd, beta, rho, q, 1.0, u0d, w0d, mode="serial")
    assert rel(_np(LVg), LV) < TOL
    assert rel(_np(LWg), LW) < TOL
    LVr, LWr = A.alif_backward(Id, Ud, Wd, None, GSd, beta, rho, q, 1.0, u0d, w0d, mode="serial")
    assert torch.equal(LVr, LVg) and torch.equal(LWr, LWg)
    LVp, _, lw1, sums = A._alif_bwd(Id, u0d, w0d, Ud, Wd, None, GSd, beta, rho, q, 1.0, 4.0, False, True)
    assert torch.equal(LVp, LVg)
    assert rel(_np(lw1), lwm1) < TOL
    got = sums.sum(dim=(1, 2)).cpu().numpy()
    for i in range(4):
        assert _param_close(float(got[i]), pg[i], sc[i]), (i, got[i], pg[i])
    # the two-level form over chunks (composed maps, carry, replay)
    LVs, LWs = A.alif_backward(Id, Ud, Wd, Sd, GSd, beta, rho, q, 1.0, u0d, w0d, mode="scan", C=T // 8, D=1)
    assert rel(_np(LVs), LV) < TOL
    assert rel(_np(LWs), LW) < TOL
    LVc, _, lwc, sc_sums = A._alif_bwd(Id, u0d, w0d, Ud, Wd, None, GSd, beta, rho, q, 1.0, 4.0, False, True,
                                       chunked=True)
    assert rel(_np(LVc), LV) < TOL
    assert rel(_np(lwc), lwm1) < TOL
    got = sc_sums.sum(dim=(1, 2)).cpu().numpy()
    for i in range(4):
        assert _param_close(float(got[i]), pg[i], sc[i]), (i, got[i], pg[i])


@pytest.mark.parametrize("fwd", ("serial", "scan"))
@pytest.mark.parametrize("T,N", ((16384, 8), (2048, 1024)))
def test_alif_layer_grads(cuda, fwd, T, N):
    """alif()'s gradients for I, u0, w0, beta, rho, q, theta0 against the oracle
    (the reference's gradient test draws x ~ N(0.06, 0.15^2), T = 4096, N = 8;
    tests/test_alif_grad.py:10-13)."""
    from hard_resets_compose_b200 import alif as A
    beta, rho, q, theta0 = 0.95, 0.995, 0.9, 1.0
    rng = np.random.default_rng(11)
    I = (0.06 + 0.15 * rng.standard_normal((T, N))).astype(np.float32)
    u0 = (0.1 * rng.standard_normal(N)).astype(np.float32)
    w0 = (0.1 * rng.random(N)).astype(np.float32)
    GS = rng.standard_normal((T, N)).astype(np.float32)
    U, W, S = O.alif_serial_forward(I, beta, rho, q, theta0, 0.0, u0, w0)
    LV, LW, lwm1, _ = O.alif_serial_backward(I, u0, w0, U, W, S, GS, beta, rho, q, theta0, 4.0)
    _, _, _, pg = O.alif_serial_backward(I, u0, w0, U, W, S, GS, beta, rho, q, theta0, 4.0, double=True)
    sc = _scales(I, u0, w0, U, W, S, GS, LV, LW, beta, q, theta0)
    Id, u0d, w0d, GSd = to_dev(cuda, I, u0, w0, GS)
    Id.requires_grad_(True)
    u0d.requires_grad_(True)
    w0d.requires_grad_(True)
    ps = [torch.tensor(v, device=cuda, requires_grad=True) for v in (beta, rho, q, theta0)]
    Sg, Ug, Wg = A.alif(Id, u0d, w0d, ps[0], ps[1], ps[2], ps[3], fwd=fwd, bwd="scan", C=128)
    torch.autograd.backward(Sg, GSd)
    assert_bit_equal(_np(Sg), S, "S")
    assert_bit_equal(_np(Ug), U, "U")
    assert_bit_equal(_np(Wg), W, "W")
    assert rel(_np(Id.grad), LV) < TOL
    assert rel(_np(u0d.grad), beta * LV[0]) < TOL
    assert rel(_np(w0d.grad), lwm1) < TOL
    for i in range(4):
        assert _param_close(float(ps[i].grad), pg[i], sc[i]), (i, float(ps[i].grad), pg[i])


def test_alif_warm_from_states(cuda):
    """alif_warm_predict from given chunk-entry states (UI, WI)."""
    from hard_resets_compose_b200 import alif as A
    T, N, C = 4096, 64, 128
    I, u0, w0 = _gen(T, N, 0.95, 2.0, seed=2)
    U, W, _ = O.alif_serial_forward(I, 0.95, 0.995, 0.9, 1.0, 0.0, u0, w0)
    UI = np.concatenate([u0[None], U[C - 1:-1:C]], 0)
    WI = np.concatenate([w0[None], W[C - 1:-1:C]], 0) * np.float32(1.01)
    want = O.alif_warm_predict(I, 0.95, 0.995, 0.9, 1.0, 0.0, u0, w0, C, Wn=3, UI=UI, WI=WI)
    Id, u0d, w0d, UId, WId = to_dev(cuda, I, u0, w0, UI.astype(np.float32), WI.astype(np.float32))
    got = A.alif_warm_predict(Id, 0.95, 0.995, 0.9, 1.0, 0.0, u0d, w0d, C, Wn=3, UI=UId, WI=WId)
    assert_bit_equal(_np(got), want, "WP")


def test_alif_argument_errors(cuda):
    from hard_resets_compose_b200 import alif as A
    I, u0, w0 = to_dev(cuda, *_gen(256, 8, 0.9, 1.0, seed=0))
    with pytest.raises(AssertionError):
        A.alif_scan_forward(I, 0.9, 0.95, 0.5, 1.0, 0.0, u0, w0, None, 0.1, C=100)
    with pytest.raises(AssertionError):
        A.alif_backward(I, I, I, None, I, 0.9, 0.95, 0.5, 1.0, u0, w0, mode="scan", C=100)
    with pytest.raises(ValueError):
        A.alif_warm_predict(I, 0.9, 0.95, 0.5, 1.0, 0.0, u0, w0, 100)
    with pytest.raises(ValueError):
        A.alif_serial_forward(I, 0.9, 0.95, 0.5, 1.0, 0.0, u0, w0[:4])
    U, W, S = A.alif_serial_forward(I[:0], 0.9, 0.95, 0.5, 1.0, 0.0, u0, w0)
    assert U.shape == W.shape == S.shape == (0, 8)
