"""Config 4 at its full length through the drop-in layer: T = 2^20 rows,
B*N = 1024 neurons, x ~ N(0.02, 0.1^2), beta = 0.99, upstream gradient
N(0, 1) on the spikes.  lif_tuned (mode "scan", the library's long-sequence
policy: speculative segments forward, chunked adjoint with its fix-up)
against the CPU oracle's serial recurrence and adjoint (oracle/lif_oracle.c,
pinned to lifscan/fast.py:69-81 and :227-239): U and S bit-identical, dI
and du0 within 1e-5 relative."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_bit_equal, gen, rel

pytestmark = pytest.mark.gpu

TOL = 1e-5


def test_lif_tuned_c4_full_length(cuda):
    from hard_resets_compose_b200 import lifscan as L
    T, N, beta = 1 << 20, 1024, 0.99
    I, u0, GS = gen(T, N, 0.02, 0.1, seed=4, grad=True)
    Us, Ss = O.serial_forward(I, beta, 1.0, 0.0, u0)
    dI_ref = O.serial_backward(I, u0, Us, Ss, GS, None, beta, 1.0, 0.0, 4.0, True)
    Id = torch.from_numpy(I).to(cuda)
    u0d = torch.from_numpy(u0).to(cuda)
    # the forward lif_tuned runs at this shape, with its potentials
    assert L.spec_segment(T, N)[0] < T, "config 4 should take the segmented forward"
    U, S = L.scan_forward_auto(Id, beta, 1.0, 0.0, u0d)
    assert_bit_equal(U.cpu().numpy(), Us, "U")
    del U
    assert_bit_equal(S.cpu().numpy(), Ss, "S (scan_forward_auto)")
    del S, Us
    Iq = Id.requires_grad_(True)
    u0q = u0d.clone().requires_grad_(True)
    S = L.lif_tuned(Iq, u0q, beta=beta, mode="scan")
    assert_bit_equal(S.detach().cpu().numpy(), Ss, "S (lif_tuned)")
    GSd = torch.from_numpy(GS).to(cuda)
    torch.autograd.backward(S, GSd)
    del S, GSd
    assert rel(Iq.grad.cpu().numpy(), dI_ref) < TOL
    assert rel(u0q.grad.cpu().numpy(), np.float32(beta) * dI_ref[0]) < TOL
