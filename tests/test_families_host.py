"""Host-side logic of the soft, affine and ALIF families (no GPU needed): the
product path refuses CPU tensors instead of falling back, the reference's
argument checks are kept, and the ALIF adjoint's chunk policy."""
import numpy as np
import pytest
import torch

from hard_resets_compose_b200 import affine as A
from hard_resets_compose_b200 import alif as AL
from hard_resets_compose_b200 import lifscan as L
from hard_resets_compose_b200 import soft as TS


def _cpu(T=64, N=8):
    g = torch.Generator().manual_seed(0)
    return torch.randn(T, N, generator=g), torch.zeros(N), torch.zeros(N)


def test_cpu_tensors_are_refused():
    """There is no CPU path: every family raises on host tensors."""
    I, u0, w0 = _cpu()
    for call in (lambda: A.aff_serial_forward(I, 0.9, 1.0, 0.3, -0.1, u0),
                 lambda: A.aff_scan_forward(I, 0.9, 1.0, 0.3, -0.1, u0, C=32),
                 lambda: A.reverse_affine_scan(I, I),
                 lambda: TS.soft_scan_forward(I, 0.9, 1.0, u0),
                 lambda: AL.alif_serial_forward(I, 0.9, 0.95, 0.5, 1.0, 0.0, u0, w0),
                 lambda: AL.alif_scan_forward(I, 0.9, 0.95, 0.5, 1.0, 0.0, u0, w0, None, 0.1, C=32),
                 lambda: AL.alif_warm_predict(I, 0.9, 0.95, 0.5, 1.0, 0.0, u0, w0, 32)):
        with pytest.raises(RuntimeError, match="CUDA"):
            call()


def test_reference_argument_checks():
    """The reference asserts T % C == 0 and 0 <= gamma <= 1 (triton_affine.py:167)
    and T % C == 0, C % D == 0 (triton_alif.py:308, :505): checked before any
    device work."""
    I, u0, w0 = _cpu()
    with pytest.raises(AssertionError):
        A.aff_scan_forward(I, 0.9, 1.0, 0.3, -0.1, u0, C=48)
    with pytest.raises(AssertionError):
        AL.alif_scan_forward(I, 0.9, 0.95, 0.5, 1.0, 0.0, u0, w0, None, 0.1, C=32, D=3)
    with pytest.raises(AssertionError):
        AL.alif_backward(I, I, I, None, I, 0.9, 0.95, 0.5, 1.0, u0, w0, mode="scan", C=48)
    with pytest.raises(ValueError):
        AL.alif_backward(I, I, I, None, I, 0.9, 0.95, 0.5, 1.0, u0, w0, mode="bogus")


@pytest.mark.parametrize("T", (1, 256, 1000, 3000, 4096, 1 << 14, 1 << 18, 1 << 20, 3 * (1 << 12)))
@pytest.mark.parametrize("N", (1, 8, 100, 1024, 16384, 100000))
def test_alif_chunk_policy(T, N):
    """Chunks divide T, and are at least ALIF_MIN_CHUNK rows unless T's factors
    forbid it; one chunk when N fills the GPU."""
    C = AL._alif_chunk(T, N)
    assert 1 <= C <= T and T % C == 0
    if C < AL.ALIF_MIN_CHUNK and C < T:
        assert T % (2 * C) != 0
    if N >= L.SCAN_BWD_SERIAL_MIN_N:
        assert C == T


def test_host_scalars_one_read():
    """Tensor parameters are read together; numbers pass through."""
    vals = L._host_scalars(torch.tensor(0.5), 1.0, torch.tensor([0.25]), 3)
    assert vals == (0.5, 1.0, 0.25, 3.0)
    assert all(isinstance(v, float) for v in vals)
    assert np.isclose(L._host_scalars(torch.tensor(0.1, dtype=torch.float64))[0], 0.1)
