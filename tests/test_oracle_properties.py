"""Oracle self-consistency on the reference's own test grids (CPU only).

Mirrors lifscan tests/test_fast.py (check_pruned: beta x drift x K, bit-exact
after repair), tests/test_triton.py:10-26 (36 configs) at reduced size, and
experiments/test_v4.py:6-20, all against the oracle's serial recurrence."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import assert_bit_equal, gen, rel

BETAS = (0.5, 0.9, 0.99, 1.0)
DRIFTS = ((0.15, 0.4), (-0.1, 0.6), (0.4, 0.2))


@pytest.mark.parametrize("beta", BETAS)
@pytest.mark.parametrize("mu,sd", DRIFTS)
@pytest.mark.parametrize("K", (2, 4, 16, 64))
def test_v3_exact_after_repair(beta, mu, sd, K):
    I, u0 = gen(1024, 96, mu, sd, seed=3, u0_sd=0.3)
    Us, Ss = O.serial_forward(I, beta, 1.0, -0.1, u0)
    U, S, st = O.scan_forward_v3(I, beta, 1.0, -0.1, u0, C=64, K=K)
    assert_bit_equal(U, Us, "U")
    assert_bit_equal(S, Ss, "S")
    assert st["repair_iters"] <= 1024 // 64
    U0, S0, _ = O.scan_forward_v3(I, beta, 1.0, -0.1, u0, C=64, K=K, repair=0)
    assert (S0 == Ss).mean() > 0.99


@pytest.mark.parametrize("beta", BETAS)
@pytest.mark.parametrize("mu,sd", DRIFTS)
@pytest.mark.parametrize("K,K2", ((16, 32), (8, 16), (2, 4)))
def test_v4_exact_after_repair(beta, mu, sd, K, K2):
    I, u0 = gen(2048, 40, mu, sd, seed=4, u0_sd=0.3)
    Us, Ss = O.serial_forward(I, beta, 1.0, -0.1, u0)
    U, S, st = O.scan_forward_v4(I, beta, 1.0, -0.1, u0, C=32, G=8, K=K, K2=K2)
    assert_bit_equal(U, Us, "U")
    assert_bit_equal(S, Ss, "S")


@pytest.mark.parametrize("detach", (True, False))
@pytest.mark.parametrize("C", (8, 64, 256))
def test_scan_backward_matches_serial(detach, C):
    I, u0, GS = gen(512, 64, 0.15, 0.4, seed=5, u0_sd=0.2, grad=True)
    U, S = O.serial_forward(I, 0.9, 1.0, -0.1, u0)
    GU = np.random.default_rng(1).standard_normal(I.shape).astype(np.float32) if not detach else None
    L1 = O.serial_backward(I, u0, U, S, GS, GU, 0.9, 1.0, -0.1, 4.0, detach)
    L2 = O.scan_backward(I, u0, U, S, GS, GU, 0.9, 1.0, -0.1, 4.0, detach, C=C)
    assert rel(L2, L1) < 1e-6


def test_edge_shapes():
    # one neuron, one chunk, capacity 1
    I, u0 = gen(64, 1, 0.3, 0.5, seed=6)
    Us, Ss = O.serial_forward(I, 0.9, 1.0, 0.0, u0)
    U, S, _ = O.scan_forward_v3(I, 0.9, 1.0, 0.0, u0, C=64, K=1)
    assert_bit_equal(U, Us, "U")
    # chunk length 1 (every step is a chunk)
    U, S, _ = O.scan_forward_v3(I, 0.9, 1.0, 0.0, u0, C=1, K=1)
    assert_bit_equal(U, Us, "U C=1")
    # T not a multiple of C is rejected
    with pytest.raises(ValueError):
        O.scan_forward_v3(I, 0.9, 1.0, 0.0, u0, C=48, K=4)
