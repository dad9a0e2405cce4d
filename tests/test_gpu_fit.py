"""Parameter gradients of the fitting layer (lifscan/fit.py:15-56) through
the C ABI: dL/dbeta, dL/dtheta, dL/du_r against the reference's formulas
evaluated in fp64 on the oracle's forward and adjoint (the oracle restates
fast.py's serial recurrence and adjoint), plus the usual dI and du0."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_bit_equal, gen, rel, to_dev

pytestmark = pytest.mark.gpu


def _ref_param_grads(I, u0, U, S, GS, Lam, beta, theta, alpha):
    """fit.py:40-46 in fp64 (terms and the sum of their magnitudes)."""
    up = np.concatenate([u0[None], U[:-1]], 0).astype(np.float64)
    v = (np.float32(beta) * np.concatenate([u0[None], U[:-1]], 0) + I).astype(np.float32).astype(np.float64)
    sig = 1.0 / (1.0 + np.exp(-alpha * (v - theta)))
    sg = alpha * sig * (1 - sig)
    lam = Lam.astype(np.float64)
    lam_next = np.concatenate([lam[1:], np.zeros_like(lam[:1])], 0)
    terms = (lam * up, -(GS * sg), S * beta * lam_next)
    return [t.sum() for t in terms], [np.abs(t).sum() for t in terms]


@pytest.mark.parametrize("mode", ("auto", "scan", "serial"))
@pytest.mark.parametrize("T,N,beta,mu,sd", ((4096, 64, 0.9, 0.15, 0.4), (2048, 1000, 0.99, 0.05, 0.2),
                                            (1 << 17, 16, 0.99, 0.02, 0.1)))
def test_param_grads_match_reference_formulas(cuda, mode, T, N, beta, mu, sd):
    from hard_resets_compose_b200 import fit
    theta, u_r, alpha = 1.0, 0.0, 4.0
    I, u0, GS = gen(T, N, mu, sd, seed=31, u0_sd=0.2, grad=True)
    U, S = O.serial_forward(I, beta, theta, u_r, u0)
    Lam = O.serial_backward(I, u0, U, S, GS, None, beta, theta, u_r, alpha, True)
    sums, mags = _ref_param_grads(I, u0, U, S, GS, Lam, beta, theta, alpha)
    Id, u0d, GSd = to_dev(cuda, I, u0, GS)
    Id.requires_grad_(True)
    u0d.requires_grad_(True)
    pb = torch.tensor(beta, device=cuda, requires_grad=True)
    pt = torch.tensor(theta, device=cuda, requires_grad=True)
    pr = torch.tensor(u_r, device=cuda, requires_grad=True)
    Sd = fit.lif_param(Id, u0d, pb, pt, pr, alpha=alpha, mode=mode)
    torch.autograd.backward(Sd, GSd)
    assert_bit_equal(Sd.detach().cpu().numpy(), S, "S")
    assert rel(Id.grad.cpu().numpy(), Lam) < 1e-5
    assert rel(u0d.grad.cpu().numpy(), beta * Lam[0]) < 1e-5
    for got, want, mag, name in zip((pb.grad, pt.grad, pr.grad), sums, mags, ("beta", "theta", "u_r")):
        assert abs(float(got) - want) <= 1e-5 * max(mag, 1e-30), (name, float(got), want, mag)


def test_param_grads_chunking_is_invariant(cuda):
    """The fp64 partial sums do not depend on how rows are chunked."""
    from hard_resets_compose_b200 import _lib
    T, N = 3000, 96
    I, u0, GS = gen(T, N, 0.1, 0.3, seed=2, grad=True)
    U, S = O.serial_forward(I, 0.95, 1.0, 0.0, u0)
    Lam = O.serial_backward(I, u0, U, S, GS, None, 0.95, 1.0, 0.0, 4.0, True)
    d = to_dev(cuda, I, u0, U, GS, Lam)
    lib = _lib.load()
    out = []
    for M in (1, 7, 64, 3000):
        part = torch.zeros(3, M, N, dtype=torch.float64, device=cuda)
        _lib.check(lib.lifb_param_grad_partials(*[_lib.ptr(t) for t in d], _lib.ptr(part), T, N, 0.95, 1.0, 4.0, M,
                                                _lib.stream_of(d[0])), "partials")
        out.append(part.sum(dim=(1, 2)).cpu().numpy())
    for o in out[1:]:
        np.testing.assert_allclose(o, out[0], rtol=1e-12, atol=1e-12)
