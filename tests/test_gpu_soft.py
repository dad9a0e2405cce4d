"""Soft-reset LIF (subtractive reset) on the GPU through the C ABI: forward
bit-identical to the reference's fp32 soft recurrence (stored outputs of its
serial kernel and exact interval-map scan, tests/golden/soft_*.npz, and the
oracle that those pin), adjoints within 1e-5 of its fp32 serial adjoint and
its float64 FFT adjoint, and the fitting layers' gradients (lifscan/fit.py:
93-154).  Grids follow tests/test_soft_scan.py:7-16 and test_soft_scan_grad.py."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_bit_equal, gen, rel, to_dev

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
TOL = 1e-5


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "soft_*.npz"))), ids=os.path.basename)
def test_soft_golden(cuda, path):
    from hard_resets_compose_b200 import lifscan as L
    from hard_resets_compose_b200 import soft as TS
    z = np.load(path)
    beta, theta, alpha, C, K = (float(v) for v in z["params"])
    Id, u0d, GSd, Ud, Vd = to_dev(cuda, z["I"], z["u0"], z["GS"], z["U"], z["V"])
    for U, S in (TS.soft_serial_forward(Id, beta, theta, u0d), TS.soft_serial_forward_tiled(Id, beta, theta, u0d),
                 TS.soft_scan_forward(Id, beta, theta, u0d, C=int(C), K=int(K), repair=10 ** 6)):
        assert_bit_equal(_np(U), z["U"], "U")
        assert_bit_equal(_np(S), z["S"], "S")
    assert rel(_np(L.soft_serial_backward(Id, u0d, Ud, GSd, beta, theta, alpha)), z["Lam_serial"]) < TOL
    assert rel(_np(TS.soft_adjoint_fft(Vd, GSd, beta, theta, alpha)), z["Lam_fft"]) < TOL


@pytest.mark.parametrize("beta", (0.9, 0.95, 0.97, 0.99))
@pytest.mark.parametrize("mu,sd", ((0.15, 0.4), (-0.1, 0.6), (0.4, 0.3)))
def test_soft_scan_bit_exact(cuda, beta, mu, sd):
    """Speculative soft scan at lengths where segments and lead-ins apply."""
    from hard_resets_compose_b200 import soft as TS
    T, N = 1 << 16, 1024
    I, u0 = gen(T, N, mu, sd, seed=2, u0_sd=0.3)
    Us, Ss = O.soft_serial_forward(I, beta, 1.0, u0)
    Id, u0d = to_dev(cuda, I, u0)
    st = {}
    U, S = TS.soft_scan_forward(Id, beta, 1.0, u0d, stats=st)
    assert st["segments"] > 1
    assert_bit_equal(_np(S), Ss, "S")
    assert_bit_equal(_np(U), Us, "U")


@pytest.mark.parametrize("N,T,beta", ((256, 1 << 15, 1.0), (333, 8192, 0.95), (1000, 1 << 14, 0.99)))
def test_soft_scan_hard_cases(cuda, N, T, beta):
    """beta = 1 (no decay: a wrong start never rejoins, the fix-up carries every
    segment), N % 4 != 0 (the plain-kernel path)."""
    from hard_resets_compose_b200 import soft as TS
    I, u0 = gen(T, N, 0.05, 0.3, seed=4, u0_sd=0.3)
    Us, Ss = O.soft_serial_forward(I, beta, 1.0, u0)
    Id, u0d = to_dev(cuda, I, u0)
    U, S = TS.soft_scan_forward(Id, beta, 1.0, u0d)
    assert_bit_equal(_np(S), Ss, "S")
    assert_bit_equal(_np(U), Us, "U")


@pytest.mark.parametrize("fn", ("lif_soft", "lif_soft_scan_serial", "lif_soft_scan"))
@pytest.mark.parametrize("T,N", ((16384, 8), (4096, 1024)))
def test_soft_fit_layers(cuda, fn, T, N):
    """Gradients of the soft fitting layers for I, u0 and beta against the
    oracle's adjoint and sum_t lam_t u_{t-1} in fp64 (lifscan/fit.py:116, :149)."""
    from hard_resets_compose_b200 import fit
    beta, theta, alpha = 0.95, 1.0, 4.0
    I, u0, GS = gen(T, N, 0.06, 0.3, seed=8, u0_sd=0.2, grad=True)
    Us, Ss = O.soft_serial_forward(I, beta, theta, u0)
    lam = O.soft_serial_backward(I, u0, Us, GS, beta, theta, alpha)
    up = np.concatenate([u0[None], Us[:-1]], 0).astype(np.float64)
    terms = lam.astype(np.float64) * up
    Id, u0d, GSd = to_dev(cuda, I, u0, GS)
    Id.requires_grad_(True)
    u0d.requires_grad_(True)
    b = torch.tensor(beta, device=cuda, requires_grad=True)
    if fn == "lif_soft":
        S = fit.lif_soft(Id, u0d, b, theta, alpha)
    else:
        S = fit.lif_soft_scan(Id, u0d, b, theta, alpha, mode="scan" if fn == "lif_soft_scan" else "serial")
    torch.autograd.backward(S, GSd)
    assert_bit_equal(_np(S), Ss, "S")
    assert rel(_np(Id.grad), lam) < TOL
    assert rel(_np(u0d.grad), beta * lam[0]) < TOL
    assert abs(float(b.grad) - terms.sum()) <= TOL * np.abs(terms).sum()
