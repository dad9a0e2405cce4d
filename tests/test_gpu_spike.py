"""The spike-input Linear kernels (lifb_spike_mask, lifb_spike_linear_lif_fwd,
lifb_spike_linear_wgrad) against plain torch on the same device: the mask bit
for bit against a torch restatement of the format, the fused forward's V and
S bit for bit against the LIF over the input-order fp32 sum (and over
nn.Linear's cuBLAS GEMM at the network's layer shapes), the sparse weight and
bias gradients within 1e-5 relative of an fp64 dI^T X and dI.sum(0), and run
to run bit-identical."""
import math

import pytest
import torch
import torch.nn as nn

from tests.helpers import rel

pytestmark = pytest.mark.gpu


def torch_mask(x2d, stride):
    """The spike mask format restated in torch: bit q of word k set where
    x[:, 32k + q] != 0, word ceil(D/32) = 1 on rows holding a nonzero value
    other than 1.0, zero padding up to `stride` words."""
    R, D = x2d.shape
    nw = (D + 31) // 32
    nz = torch.zeros(R, nw * 32, dtype=torch.int64, device=x2d.device)
    nz[:, :D] = (x2d != 0).long()
    w = (nz.view(R, nw, 32) << torch.arange(32, device=x2d.device)).sum(2)
    w = torch.where(w >= 2 ** 31, w - 2 ** 32, w)
    out = torch.zeros(R, stride, dtype=torch.int64, device=x2d.device)
    out[:, :nw] = w
    out[:, nw] = ((x2d != 0) & (x2d != 1)).any(1).long()
    return out.to(torch.int32)


def raster(shape, rate, device, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.rand(shape, generator=g) < rate).float().to(device)


@pytest.mark.parametrize("R,D", ((1, 1), (37, 31), (1000, 700), (513, 256), (65, 1024), (3, 33)))
def test_spike_mask_matches_format(cuda, R, D):
    from hard_resets_compose_b200 import _lib
    from hard_resets_compose_b200.shdnet import spike_mask
    x = raster((R, D), 0.1, cuda, seed=R + D)
    if R > 2:
        x[1, D // 2] = 0.5            # an odd row
        x[2, 0] = float("nan")        # NaN counts as nonzero and odd
        x[2, D - 1] = -0.0            # -0 is zero
    m = spike_mask(x)
    assert m.shape == (R, _lib.load().lifb_spike_mask_stride(D))
    assert torch.equal(m, torch_mask(x, m.shape[1]))


def seq_linear(x2d, W, b):
    """x W^T + b summed in input order from 0 with the bias added last, for a
    0/1 input (each term x_c * W[j, c] is exact, each add rounds once: the
    order of a sequential fp32 GEMM)."""
    acc = torch.zeros(x2d.shape[0], W.shape[0], device=x2d.device)
    for c in range(x2d.shape[1]):
        acc = acc + x2d[:, c:c + 1] * W[:, c]
    return acc + b


def _linear_then_lif(x, fc, beta):
    from hard_resets_compose_b200 import lifscan as Lm
    T, B, _ = x.shape
    I = fc(x).reshape(T, -1)
    return I, Lm.lif_tuned(I, torch.zeros(I.shape[1], device=x.device), beta=beta).reshape(T, B, -1)


@pytest.mark.parametrize("T,B,din,dout,rate,scale", ((64, 5, 700, 256, 0.03, 6.0), (33, 7, 37, 64, 0.2, 2.0),
                                                   (50, 3, 1024, 96, 0.02, 8.0), (17, 2, 256, 32, 0.3, 1.5),
                                                   (40, 6, 256, 256, 0.1, 3.0), (35, 73, 700, 256, 0.03, 6.0)))
def test_fused_forward_v_s_and_mask(cuda, T, B, din, dout, rate, scale):
    """V and S equal the LIF over I summed in input order (the sequential
    GEMM order), bit for bit, and so over cuBLAS's I for the network's layer
    shapes (700 -> 256, 256 -> 256, where cuBLAS sums in that order; for other
    shapes it may split the sum); the mask the fused layer writes equals
    lifb_spike_mask of its S."""
    from hard_resets_compose_b200 import _lib
    from hard_resets_compose_b200._lib import check, ptr, stream_of
    from hard_resets_compose_b200.shdnet import spike_mask
    torch.manual_seed(T + din)
    fc = nn.Linear(din, dout).to(cuda)
    with torch.no_grad():
        fc.weight.mul_(scale)
    x = raster((T, B, din), rate, cuda, seed=din)
    lib = _lib.load()
    xm = spike_mask(x.view(T * B, din))
    V = torch.empty(T, B * dout, device=cuda)
    S = torch.empty(T, B * dout, device=cuda)
    sm = torch.empty(T * B, lib.lifb_spike_mask_stride(dout), dtype=torch.int32, device=cuda)
    u0 = torch.randn(B * dout, device=cuda) * 0.3
    check(lib.lifb_spike_linear_lif_fwd(ptr(x), ptr(xm), ptr(fc.weight.detach()), ptr(fc.bias.detach()), ptr(u0),
                                        ptr(V), ptr(S), ptr(sm), T, B, din, dout, 0.9, 1.0, 0.0, stream_of(x)),
          "fwd")
    torch.cuda.synchronize()
    with torch.no_grad():
        I = seq_linear(x.view(T * B, din), fc.weight, fc.bias).reshape(T, -1)
        if (din, dout) in ((700, 256), (256, 256)):
            assert torch.equal(I, fc(x).reshape(T, -1))
        u = u0.clone()
        Vr, Sr = [], []
        for t in range(T):
            v = 0.9 * u + I[t]  # two roundings, as the kernel steps
            s = v >= 1.0
            Vr.append(v)
            Sr.append(s.float())
            u = torch.where(s, torch.zeros_like(v), v)
    assert S.sum() > 0
    assert torch.equal(V.view(torch.int32), torch.stack(Vr).view(torch.int32))
    assert torch.equal(S, torch.stack(Sr))
    assert torch.equal(sm, torch_mask(S.view(T * B, dout), sm.shape[1]))
    assert torch.equal(sm, spike_mask(S.view(T * B, dout)))


def test_fused_forward_odd_values_and_nonfinite_weights(cuda):
    """Rows with values other than 0/1 take the values from the dense input;
    a non-finite weight makes the GEMM's zero terms NaN, which the fused sum
    reproduces; S stays bit-equal to the unfused layer either way (the
    network's first layer shape, where cuBLAS sums in input order)."""
    from hard_resets_compose_b200.shdnet import spike_linear_lif
    T, B, din, dout = 64, 5, 700, 256
    torch.manual_seed(1)
    fc = nn.Linear(din, dout).to(cuda)
    with torch.no_grad():
        fc.weight.mul_(5.0)
    x = raster((T, B, din), 0.05, cuda, seed=5)
    x[3, 1, 7] = 0.25
    x[10, 0, 100] = -2.0
    x[11, 2, :] = 0.5 * x[11, 2, :]
    x[12, 4, 650] = float("nan")
    S = spike_linear_lif(x, fc.weight, fc.bias, 0.9)
    _, S2 = _linear_then_lif(x, fc, 0.9)
    assert torch.equal(S.detach(), S2.detach())
    with torch.no_grad():
        fc.weight[5, 17] = float("inf")
        fc.weight[40, 3] = float("nan")
    S = spike_linear_lif(x, fc.weight, fc.bias, 0.9)
    _, S2 = _linear_then_lif(x, fc, 0.9)
    assert torch.equal(S.detach(), S2.detach())


@pytest.mark.parametrize("R,din,dout,rate", ((65536, 700, 256, 0.0225), (4100, 256, 256, 0.1), (2049, 37, 64, 0.3),
                                            (31, 1024, 32, 0.05), (5000, 100, 96, 0.0), (65536, 256, 20, 0.12),
                                            (700, 50, 4, 0.2)))
def test_wgrad_matches_torch(cuda, R, din, dout, rate):
    """gW = dI^T X and gb = dI.sum(0) over the active inputs only, within 1e-5
    of torch's fp32 GEMM and sum; bit-identical from run to run."""
    from hard_resets_compose_b200 import _lib
    from hard_resets_compose_b200._lib import check, ptr, stream_of
    from hard_resets_compose_b200.shdnet import spike_mask
    lib = _lib.load()
    x = raster((R, din), rate, cuda, seed=R)
    if R > 40:
        x[40, : min(din, 50)] *= 0.75  # an odd row
    dI = torch.randn(R, dout, device=cuda)
    m = spike_mask(x)
    ws = torch.empty(lib.lifb_spike_linear_wgrad_workspace_bytes(R, din, dout), dtype=torch.uint8, device=cuda)
    outs = []
    for _ in range(2):
        gw = torch.full((dout, din), float("nan"), device=cuda)
        gb = torch.full((dout,), float("nan"), device=cuda)
        check(lib.lifb_spike_linear_wgrad(ptr(dI), ptr(x), ptr(m), ptr(gw), ptr(gb), R, din, dout, ptr(ws),
                                          ws.numel(), stream_of(x)), "wgrad")
        outs.append((gw, gb))
    torch.cuda.synchronize()
    ref_w = dI.double().t().mm(x.double()).float()
    ref_b = dI.double().sum(0).float()
    gw, gb = outs[0]
    assert torch.isfinite(gw).all() and torch.isfinite(gb).all()
    scale_w = max(float(ref_w.abs().max()), 1e-30)
    assert float((gw - ref_w).abs().max()) / scale_w < 1e-5
    assert rel(gb.cpu().numpy(), ref_b.cpu().numpy()) < 1e-5
    assert torch.equal(outs[0][0], outs[1][0]) and torch.equal(outs[0][1], outs[1][1])


def test_layer_gradients_and_mask_chain(cuda):
    """Two fused layers back to back: the second reads the first's carried
    mask (no rescan), spikes bit-equal to the unfused pair, every gradient
    within 1e-5 of it; an in-place change to the first layer's output drops
    the carried mask."""
    from hard_resets_compose_b200 import shdnet
    T, B, din, H = 128, 8, 700, 256
    torch.manual_seed(2)
    fc1, fc2 = nn.Linear(din, H).to(cuda), nn.Linear(H, H).to(cuda)
    with torch.no_grad():
        fc1.weight.mul_(6.0)
        fc2.weight.mul_(3.0)
    x = raster((T, B, din), 0.0225, cuda, seed=9)
    s1 = shdnet.spike_linear_lif(x, fc1.weight, fc1.bias, 0.9)
    assert shdnet._carried_mask(s1) is not None
    s2 = shdnet.spike_linear_lif(s1, fc2.weight, fc2.bias, 0.9)
    g = torch.randn_like(s2)
    grads = torch.autograd.grad(s2, (fc1.weight, fc1.bias, fc2.weight, fc2.bias), g)
    _, r1 = _linear_then_lif(x, fc1, 0.9)
    _, r2 = _linear_then_lif(r1, fc2, 0.9)
    rgrads = torch.autograd.grad(r2, (fc1.weight, fc1.bias, fc2.weight, fc2.bias), g)
    assert s1.sum() > 0 and s2.sum() > 0
    assert torch.equal(s1.detach(), r1.detach()) and torch.equal(s2.detach(), r2.detach())
    for a, r in zip(grads, rgrads):
        assert rel(a.cpu().numpy(), r.cpu().numpy()) < 1e-5
    with torch.no_grad():
        s1.mul_(1.0)
    assert shdnet._carried_mask(s1) is None
    assert not math.isnan(float(s2.sum()))


def test_spike_input_linear_readout(cuda):
    """The readout on a spike input: output bit-equal to nn.functional.linear,
    the gradients of x, W and b within 1e-5 of torch's, with and without a
    carried mask."""
    from hard_resets_compose_b200 import shdnet
    T, B, din, dout = 256, 16, 256, 20
    torch.manual_seed(4)
    fc = nn.Linear(din, dout).to(cuda)
    x = raster((T, B, din), 0.15, cuda, seed=11).requires_grad_(True)
    g = torch.randn(T, B, dout, device=cuda)
    y = shdnet.spike_input_linear(x, fc.weight, fc.bias)
    grads = torch.autograd.grad(y, (x, fc.weight, fc.bias), g)
    x2 = x.detach().clone().requires_grad_(True)
    y2 = nn.functional.linear(x2, fc.weight, fc.bias)
    rgrads = torch.autograd.grad(y2, (x2, fc.weight, fc.bias), g)
    assert torch.equal(y.detach(), y2.detach())
    for a, r in zip(grads, rgrads):
        assert rel(a.cpu().numpy(), r.cpu().numpy()) < 1e-5


def test_spike_kernels_empty_and_errors(cuda):
    """Empty T or B is a no-op; a bad shape is refused with a status, not run."""
    from hard_resets_compose_b200 import _lib
    from hard_resets_compose_b200._lib import ptr, stream_of
    lib = _lib.load()
    x = torch.zeros(4, 3, 64, device=cuda)
    m = torch.zeros(12, lib.lifb_spike_mask_stride(64), dtype=torch.int32, device=cuda)
    W = torch.zeros(32, 64, device=cuda)
    V = torch.zeros(4, 3 * 32, device=cuda)
    S = torch.zeros_like(V)
    s = stream_of(x)
    assert lib.lifb_spike_linear_lif_fwd(ptr(x), ptr(m), ptr(W), None, None, ptr(V), ptr(S), None, 0, 3, 64, 32,
                                         0.9, 1.0, 0.0, s) == 0
    assert lib.lifb_spike_linear_lif_fwd(ptr(x), ptr(m), ptr(W), None, None, ptr(V), ptr(S), None, 4, 0, 64, 32,
                                         0.9, 1.0, 0.0, s) == 0
    assert lib.lifb_spike_mask(ptr(x), ptr(m), 0, 64, s) == 0
    # Dout not a multiple of 32: unsupported (the caller runs the unfused layer)
    assert lib.lifb_spike_linear_lif_fwd(ptr(x), ptr(m), ptr(W), None, None, ptr(V), ptr(S), None, 4, 3, 64, 20,
                                         0.9, 1.0, 0.0, s) == 4
    # Din past 1024: unsupported mask
    assert lib.lifb_spike_mask(ptr(x), ptr(m), 12, 2000, s) == 4
    # null pointers: invalid argument
    assert lib.lifb_spike_linear_wgrad(None, ptr(x), ptr(m), ptr(W), None, 12, 64, 32, None, 0, s) == 1
    torch.cuda.synchronize()
