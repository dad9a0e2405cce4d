"""Affine-reset LIF (u <- gamma*v + delta on a spike) on the GPU through the C
ABI: forward bit-identical to the reference's serial kernel and exact map
scan (stored outputs over the (gamma, delta) x beta grid of its
tests/test_affine.py, tests/golden/affine_grid.npz, and the oracle those
pin), gradients for I, u0, beta, gamma, delta within 1e-5 of LIFAffineFn's
own backward and of the oracle (lifscan/triton_affine.py:214-246)."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_bit_equal, gen, rel, to_dev

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "affine_grid.npz")
TOL = 1e-5
GRID = ((0.0, 0.0), (0.0, -0.2), (0.3, -0.1), (0.7, -0.5), (1.0, -1.0), (0.5, 0.2))
KEYS = [f"g{g}b{b}" for g in range(6) for b in range(2)]


def _np(t):
    return t.detach().cpu().numpy()


def _param_close(got, want):
    return abs(got - want) <= TOL * (abs(want) + 1e-3)


@pytest.mark.parametrize("key", KEYS)
def test_affine_golden(cuda, key):
    from hard_resets_compose_b200 import affine as A
    z = np.load(GOLD)
    beta, theta, gamma, delta, alpha = (float(v) for v in z[f"{key}_params"])
    Id, u0d, GSd = to_dev(cuda, z[f"{key}_I"], z[f"{key}_u0"], z[f"{key}_GS"])
    for U, S in (A.aff_serial_forward(Id, beta, theta, gamma, delta, u0d),
                 A.aff_scan_forward(Id, beta, theta, gamma, delta, u0d, C=32, K=16, repair=10 ** 6)):
        assert_bit_equal(_np(U), z[f"{key}_U"], "U")
        assert_bit_equal(_np(S), z[f"{key}_S"], "S")
    dp = z[f"{key}_dp"].astype(np.float64)
    for mode in ("serial", "scan"):
        Ig = Id.clone().requires_grad_(True)
        ug = u0d.clone().requires_grad_(True)
        ps = [torch.tensor(v, device=cuda, requires_grad=True) for v in (beta, gamma, delta)]
        S = A.lif_affine(Ig, ug, ps[0], ps[1], ps[2], theta=theta, alpha=alpha, mode=mode, C=32, K=16)
        torch.autograd.backward(S, GSd)
        assert_bit_equal(_np(S), z[f"{key}_S"], "S")
        assert rel(_np(Ig.grad), z[f"{key}_dI"]) < TOL
        assert rel(_np(ug.grad), z[f"{key}_du0"]) < TOL
        for i in range(3):
            assert _param_close(float(ps[i].grad), dp[i]), (mode, i, float(ps[i].grad), dp[i])


@pytest.mark.parametrize("beta", (0.9, 0.97, 0.99))
@pytest.mark.parametrize("gamma,delta", GRID)
def test_affine_scan_bit_exact(cuda, gamma, delta, beta):
    """The speculative affine scan where segments and lead-ins apply."""
    from hard_resets_compose_b200 import affine as A
    T, N = 1 << 16, 1024
    I, u0 = gen(T, N, 0.15, 0.4, seed=11, u0_sd=0.2)
    Us, Ss = O.aff_serial_forward(I, beta, 1.0, gamma, delta, u0)
    Id, u0d = to_dev(cuda, I, u0)
    st = {}
    U, S = A.aff_scan_forward(Id, beta, 1.0, gamma, delta, u0d, stats=st)
    assert st["segments"] > 1
    assert_bit_equal(_np(S), Ss, "S")
    assert_bit_equal(_np(U), Us, "U")


@pytest.mark.parametrize("N,T,beta,gamma,delta", ((256, 1 << 15, 1.0, 1.0, -1.0), (256, 1 << 15, 1.0, 0.9, 0.05),
                                                   (333, 8192, 0.95, 0.3, -0.1), (1000, 1 << 14, 0.99, 0.7, -0.5),
                                                   (1024, 1 << 15, 0.99, 0.0, -0.3)))
def test_affine_scan_hard_cases(cuda, N, T, beta, gamma, delta):
    """beta = 1 with gamma = 1 (a wrong start never rejoins: the fix-up carries
    every segment), N % 4 != 0 (the plain-kernel path), gamma = 0 (the hard
    reset: equal to the hard-reset kernels bit for bit)."""
    from hard_resets_compose_b200 import affine as A
    from hard_resets_compose_b200 import lifscan as L
    I, u0 = gen(T, N, 0.05, 0.3, seed=4, u0_sd=0.3)
    Us, Ss = O.aff_serial_forward(I, beta, 1.0, gamma, delta, u0)
    Id, u0d = to_dev(cuda, I, u0)
    U, S = A.aff_scan_forward(Id, beta, 1.0, gamma, delta, u0d)
    assert_bit_equal(_np(S), Ss, "S")
    assert_bit_equal(_np(U), Us, "U")
    if gamma == 0.0:
        Uh, Sh = L.scan_forward_auto(Id, beta, 1.0, delta, u0d)
        assert_bit_equal(_np(Uh), Us, "U hard")
        assert_bit_equal(_np(Sh), Ss, "S hard")


def test_affine_soft_is_soft(cuda):
    """gamma = 1, delta = -theta runs the soft-reset model bit for bit."""
    from hard_resets_compose_b200 import affine as A
    from hard_resets_compose_b200 import soft as TS
    T, N = 1 << 15, 512
    I, u0 = gen(T, N, 0.15, 0.4, seed=5, u0_sd=0.3)
    Id, u0d = to_dev(cuda, I, u0)
    Ua, Sa = A.aff_scan_forward(Id, 0.97, 1.0, 1.0, -1.0, u0d)
    Us, Ss = TS.soft_scan_forward(Id, 0.97, 1.0, u0d)
    assert torch.equal(Ua, Us) and torch.equal(Sa, Ss)


@pytest.mark.parametrize("mode", ("serial", "scan"))
@pytest.mark.parametrize("T,N", ((16384, 8), (4096, 1024), (2048, 333)))
@pytest.mark.parametrize("gamma,delta", ((0.4, -0.3), (1.0, -1.0), (0.0, 0.1)))
def test_affine_grads(cuda, mode, T, N, gamma, delta):
    """lif_affine's gradients for I, u0, beta, gamma, delta against the oracle
    (fp32 adjoint in order, parameter sums in fp64)."""
    from hard_resets_compose_b200 import affine as A
    beta, theta, alpha = 0.95, 1.0, 4.0
    I, u0, GS = gen(T, N, 0.08, 0.35, seed=9, u0_sd=0.2, grad=True)
    Us, Ss = O.aff_serial_forward(I, beta, theta, gamma, delta, u0)
    lam, pg = O.aff_serial_backward(I, u0, Us, GS, beta, theta, gamma, alpha)
    Id, u0d, GSd = to_dev(cuda, I, u0, GS)
    Id.requires_grad_(True)
    u0d.requires_grad_(True)
    ps = [torch.tensor(v, device=cuda, requires_grad=True) for v in (beta, gamma, delta)]
    S = A.lif_affine(Id, u0d, ps[0], ps[1], ps[2], theta=theta, alpha=alpha, mode=mode)
    torch.autograd.backward(S, GSd)
    assert_bit_equal(_np(S), Ss, "S")
    assert rel(_np(Id.grad), lam) < TOL
    assert rel(_np(u0d.grad), beta * lam[0]) < TOL
    for i in range(3):
        assert _param_close(float(ps[i].grad), pg[i]), (i, float(ps[i].grad), pg[i])


def test_affine_float_params_get_no_grad(cuda):
    """Parameters passed as Python numbers: only I and u0 receive gradients."""
    from hard_resets_compose_b200 import affine as A
    I, u0, GS = gen(1024, 64, 0.1, 0.4, seed=1, u0_sd=0.2, grad=True)
    Id, u0d, GSd = to_dev(cuda, I, u0, GS)
    Id.requires_grad_(True)
    S = A.lif_affine(Id, u0d, 0.9, 0.5, -0.2, mode="serial")
    torch.autograd.backward(S, GSd)
    Us, _ = O.aff_serial_forward(I, 0.9, 1.0, 0.5, -0.2, u0)
    lam, _ = O.aff_serial_backward(I, u0, Us, GS, 0.9, 1.0, 0.5, 4.0)
    assert rel(_np(Id.grad), lam) < TOL


@pytest.mark.parametrize("shape", ((1,), (777,), (513, 7), (64, 3, 5)))
def test_reverse_affine_scan(cuda, shape):
    """lam_t = a_t lam_{t+1} + b_t, lam_T = 0 (lifscan/triton_affine.py:202-211),
    against the same recurrence in fp32 in order on the CPU."""
    from hard_resets_compose_b200 import affine as A
    rng = np.random.default_rng(7)
    a = rng.uniform(0.0, 1.0, shape).astype(np.float32)
    b = rng.standard_normal(shape).astype(np.float32)
    want = np.empty_like(b)
    acc = np.zeros(shape[1:], np.float32)
    for t in range(shape[0] - 1, -1, -1):
        acc = (a[t] * acc).astype(np.float32) + b[t]
        want[t] = acc
    got = A.reverse_affine_scan(*to_dev(cuda, a, b))
    assert got.shape == a.shape
    assert_bit_equal(_np(got), want, "reverse scan")


def test_affine_argument_errors(cuda):
    from hard_resets_compose_b200 import affine as A
    I, u0 = to_dev(cuda, *gen(256, 8, 0.1, 0.3, seed=0, u0_sd=0.1))
    with pytest.raises(AssertionError):
        A.aff_scan_forward(I, 0.9, 1.0, 1.5, 0.0, u0)
    with pytest.raises(AssertionError):
        A.aff_scan_forward(I, 0.9, 1.0, -0.1, 0.0, u0)
    with pytest.raises(AssertionError):
        A.aff_scan_forward(I, 0.9, 1.0, 0.5, 0.0, u0, C=100)
    U, S = A.aff_scan_forward(I[:0], 0.9, 1.0, 0.5, 0.0, u0)
    assert U.shape == (0, 8) and S.shape == (0, 8)


@pytest.mark.parametrize("T,N", ((1024, 16384), (3000, 333), (16384, 8)))
def test_affine_vpath(cuda, T, N):
    """The layer's single-pass path: V (the potentials before the reset) bit for
    bit, and the adjoint from V with the beta, gamma, delta sums fused into the
    same sweep (TMA kernel for N % 4 == 0, plain kernel otherwise)."""
    from hard_resets_compose_b200 import affine as A
    beta, theta, gamma, delta, alpha = 0.97, 1.0, 0.6, -0.25, 4.0
    I, u0, GS = gen(T, N, 0.08, 0.35, seed=13, u0_sd=0.2, grad=True)
    Us, Ss, Vs = O.aff_serial_forward(I, beta, theta, gamma, delta, u0, want_v=True)
    lam, pg = O.aff_serial_backward(I, u0, Us, GS, beta, theta, gamma, alpha)
    Id, u0d, GSd = to_dev(cuda, I, u0, GS)
    V, S = A.aff_serial_forward_v(Id, beta, theta, gamma, delta, u0d)
    assert_bit_equal(_np(V), Vs, "V")
    assert_bit_equal(_np(S), Ss, "S")
    Lam, got = A.aff_adjoint_v(V, u0d, GSd, beta, theta, gamma, delta, alpha)
    assert rel(_np(Lam), lam) < TOL
    for i in range(3):
        assert _param_close(float(got[i]), pg[i]), (i, float(got[i]), pg[i])
    Lam2, none = A.aff_adjoint_v(V, u0d, GSd, beta, theta, gamma, delta, alpha, param_grads=False)
    assert none is None and torch.equal(Lam2, Lam)
