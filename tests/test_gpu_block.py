"""The block-level fused forward (csrc/scan_block.cu) through the C ABI: one
CTA per 32-neuron slab, all T rows in shared memory, every phase in one
launch.  Map mode through scan_forward_v3 without stats (the reference's
two-level scan, lifscan/triton_lif.py:782-817), lead-in mode through
scan_forward_spec with short segments.  U and S must be bit-identical to the
serial recurrence (the CPU oracle, pinned to lifscan/fast.py:69-81) on the
grid of the reference's GPU tests (tests/test_triton.py:10-26: beta x drift x
K, u_r = -0.1, u0 ~ N(0, 0.3^2)), and each call must be one launch."""
import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import assert_bit_equal, gen, to_dev

pytestmark = pytest.mark.gpu

BETAS = (0.5, 0.9, 0.99, 1.0)
DRIFTS = ((0.15, 0.4), (-0.1, 0.6), (0.4, 0.2))


def _L():
    from hard_resets_compose_b200 import lifscan
    return lifscan


def _launches():
    from hard_resets_compose_b200 import _lib
    return _lib.load().lifb_kernel_launches()


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("beta", BETAS)
@pytest.mark.parametrize("mu,sd", DRIFTS)
@pytest.mark.parametrize("K", (1, 4, 16))
def test_block_maps_bit_exact(cuda, beta, mu, sd, K):
    """K = 1 overflows almost every map: the carry's serial fallback."""
    T, N = 1024, 1000
    I, u0 = gen(T, N, mu, sd, seed=0, u0_sd=0.3)
    Us, Ss = O.serial_forward(I, beta, 1.0, -0.1, u0)
    Id, u0d = to_dev(cuda, I, u0)
    n0 = _launches()
    U, S = _L().scan_forward_v3(Id, beta, 1.0, -0.1, u0d, C=64, K=K)
    assert _launches() - n0 == 1
    assert_bit_equal(_np(U), Us, "U")
    assert_bit_equal(_np(S), Ss, "S")


@pytest.mark.parametrize("T,C,K,N", ((512, 32, 16, 4096), (256, 16, 8, 36), (128, 64, 16, 4), (1536, 96, 4, 500),
                                     (1024, 256, 16, 64), (2048, 128, 2, 32)))
def test_block_maps_shapes(cuda, T, C, K, N):
    """Chunk counts 2-16, a chunk length that is not a power of two, partial
    slabs (N = 4, 36, 500), the largest slab that fits beside its maps."""
    from hard_resets_compose_b200 import _lib  # noqa: F401
    I, u0 = gen(T, N, 0.1, 0.3, seed=3, u0_sd=0.3)
    Us, Ss = O.serial_forward(I, 0.9, 1.0, 0.0, u0)
    Id, u0d = to_dev(cuda, I, u0)
    n0 = _launches()
    U, S = _L().scan_forward_v3(Id, 0.9, 1.0, 0.0, u0d, C=C, K=K)
    one = _launches() - n0 == 1
    assert_bit_equal(_np(U), Us, "U")
    assert_bit_equal(_np(S), Ss, "S")
    if T * 128 + (T // C) * (2 * max(K, 4) + 6) * 128 <= 200 * 1024:
        assert one


@pytest.mark.parametrize("beta", BETAS)
@pytest.mark.parametrize("mu,sd", DRIFTS)
@pytest.mark.parametrize("Lseg,W", ((64, 64), (64, 0), (32, 200), (128, 4096)))
def test_block_leadin_bit_exact(cuda, beta, mu, sd, Lseg, W):
    """Lead-in mode: W = 0 guesses u_r for every chunk (the fix-up carries
    everything); W beyond row 0 starts from u0 (exact)."""
    T, N = 1024, 1000
    I, u0 = gen(T, N, mu, sd, seed=1, u0_sd=0.3)
    Us, Ss = O.serial_forward(I, beta, 1.0, -0.1, u0)
    Id, u0d = to_dev(cuda, I, u0)
    n0 = _launches()
    U, S = _L().scan_forward_spec(Id, beta, 1.0, -0.1, u0d, L=Lseg, W=W)
    assert _launches() - n0 == 1
    assert_bit_equal(_np(U), Us, "U")
    assert_bit_equal(_np(S), Ss, "S")


def test_block_c1_full_size(cuda):
    """Config 1 (B*N = 4096, T = 1024, x ~ N(0.1, 0.3^2), beta = 0.9): both
    modes, one launch each."""
    I, u0 = gen(1024, 4096, 0.1, 0.3, seed=0)
    Us, Ss = O.serial_forward(I, 0.9, 1.0, 0.0, u0)
    Id, u0d = to_dev(cuda, I, u0)
    for fn in (lambda: _L().scan_forward_v3(Id, 0.9, 1.0, 0.0, u0d, C=64, K=16),
               lambda: _L().scan_forward_spec(Id, 0.9, 1.0, 0.0, u0d, L=64, W=64)):
        n0 = _launches()
        U, S = fn()
        assert _launches() - n0 == 1
        assert_bit_equal(_np(U), Us, "U")
        assert_bit_equal(_np(S), Ss, "S")


def test_block_falls_back_when_it_does_not_apply(cuda):
    """N % 4 != 0 (no TMA), K > 16, stats requested: the grid pipeline, still
    exact."""
    T = 1024
    for N, K, stats in ((777, 16, None), (1000, 32, None), (1000, 16, {})):
        I, u0 = gen(T, N, 0.15, 0.4, seed=5, u0_sd=0.3)
        Us, Ss = O.serial_forward(I, 0.9, 1.0, -0.1, u0)
        Id, u0d = to_dev(cuda, I, u0)
        n0 = _launches()
        U, S = _L().scan_forward_v3(Id, 0.9, 1.0, -0.1, u0d, C=64, K=K, stats=stats)
        assert _launches() - n0 > 1
        assert_bit_equal(_np(U), Us, "U")
        assert_bit_equal(_np(S), Ss, "S")
