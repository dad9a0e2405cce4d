"""Dense-layer input gradient on the tensor cores (lifb_dense_dgrad,
csrc/dgrad_tc.cu): dX = dY . W as three TF32 products accumulated in fp32,
checked against an fp64 product and torch's fp32 GEMM.  The bound is the
gradient tolerance of the layer API, 1e-5 relative (Frobenius); measured:
about 1.5e-6 at K = 256 and 3.7e-6 at K = 512 against fp64 (an fp32 SGEMM:
3e-7), the rest being the tensor cores' own fp32 accumulation along K."""
TOL = 1e-5
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from hard_resets_compose_b200 import _lib as lib
    return lib.load()


def dgrad(dY, W):
    L = _lib()
    R, Dout = dY.shape
    Din = W.shape[1]
    dX = torch.empty(R, Din, device=dY.device)
    nb = L.lifb_dense_dgrad_workspace_bytes(Din, Dout)
    ws = torch.empty(nb, dtype=torch.uint8, device=dY.device)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.lifb_dense_dgrad(dY.data_ptr(), W.data_ptr(), dX.data_ptr(), R, Din, Dout, ws.data_ptr(), nb, st)
    return rc, dX


def rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm()).item()


@pytest.mark.parametrize("R,Din,Dout", ((65536, 256, 256), (1000, 128, 64), (37, 64, 32), (384, 256, 512),
                                        (129, 256, 32), (4096, 64, 256), (300, 128, 48),
                                        (65536, 256, 20), (1000, 256, 4), (513, 64, 36)))
def test_dense_dgrad_matches_fp64(cuda, R, Din, Dout):
    g = torch.Generator(device="cuda").manual_seed(R + Din + Dout)
    dY = torch.randn(R, Dout, device="cuda", generator=g) * 1e-3
    bound = 1.0 / Dout ** 0.5
    W = (torch.rand(Dout, Din, device="cuda", generator=g) * 2 - 1) * bound
    rc, dX = dgrad(dY, W)
    torch.cuda.synchronize()
    assert rc == 0
    ref = dY.double() @ W.double()
    assert rel(dX, ref) < TOL
    assert rel(dX, dY @ W) < TOL
    # the rows past the last full tile and every column are written
    assert torch.isfinite(dX).all()


def test_dense_dgrad_spike_gradient_shape(cuda):
    """The network's case: dI of a LIF layer (mostly tiny values, a few large)."""
    g = torch.Generator(device="cuda").manual_seed(3)
    dY = torch.randn(1024 * 64, 256, device="cuda", generator=g) * 1e-4
    dY[::97] *= 1e3
    W = (torch.rand(256, 256, device="cuda", generator=g) * 2 - 1) * (1.5 / 16)
    rc, dX = dgrad(dY, W)
    torch.cuda.synchronize()
    assert rc == 0
    assert rel(dX, dY.double() @ W.double()) < TOL


def test_dense_dgrad_non_finite_stays_in_its_rows(cuda):
    """An inf or NaN in dY makes its own output row non-finite and leaves the
    other rows exact to the bound; nothing non-finite turns finite."""
    g = torch.Generator(device="cuda").manual_seed(7)
    dY = torch.randn(300, 64, device="cuda", generator=g)
    W = (torch.rand(64, 128, device="cuda", generator=g) * 2 - 1) / 8
    dY[5, 3] = float("inf")
    dY[200, 0] = float("nan")
    rc, dX = dgrad(dY, W)
    torch.cuda.synchronize()
    assert rc == 0
    bad = torch.zeros(300, dtype=torch.bool, device="cuda")
    bad[5] = bad[200] = True
    assert not torch.isfinite(dX[bad]).any()
    assert torch.isfinite(dX[~bad]).all()
    assert rel(dX[~bad], dY[~bad].double() @ W.double()) < TOL


def test_dense_dgrad_refusals(cuda):
    L = _lib()
    dY = torch.zeros(8, 18, device="cuda")
    W = torch.zeros(18, 256, device="cuda")
    rc, _ = dgrad(dY, W)
    assert rc == 4  # LIFB_ERR_UNSUPPORTED: Dout % 4 != 0
    dY = torch.zeros(8, 32, device="cuda")
    W = torch.zeros(32, 96, device="cuda")
    rc, _ = dgrad(dY, W)
    assert rc == 4  # Din not in {64, 128, 256}
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.lifb_dense_dgrad(None, None, None, 0, 64, 32, None, 0, st) == 0  # empty
    assert L.lifb_dense_dgrad(None, W.data_ptr(), None, 8, 64, 32, None, 0, st) != 0
