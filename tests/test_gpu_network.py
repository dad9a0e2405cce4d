"""The 700-256-256-20 network (config 3's consumer) on the B200 kernels
against the same network with a plain PyTorch fp32 serial LIF loop on the
same device: identical weights and GEMMs, so spikes must be bit-equal and
every parameter gradient within 1e-5 relative."""
import pytest
import torch
import torch.nn as nn

from tests.helpers import rel

pytestmark = pytest.mark.gpu


def _torch_lif(I, beta, alpha=4.0):
    """Serial hard-reset LIF in plain torch ops (beta*u and +x rounded
    separately, as lifscan/fast.py:52-66 computes it), sigmoid surrogate,
    detached reset to 0."""
    u = torch.zeros(I.shape[1], device=I.device)
    out = []
    for t in range(I.shape[0]):
        v = beta * u + I[t]
        sg = torch.sigmoid(alpha * (v - 1.0))
        s = (v >= 1.0).float() + (sg - sg.detach())
        u = v * (1.0 - s.detach())
        out.append(s)
    return torch.stack(out)


def _reference_forward(net, x):
    s1 = _torch_lif(net.l1.fc(x).reshape(x.shape[0], -1), net.l1.beta).reshape(x.shape[0], x.shape[1], -1)
    s2 = _torch_lif(net.l2.fc(s1).reshape(x.shape[0], -1), net.l2.beta).reshape(x.shape[0], x.shape[1], -1)
    z = net.out(s2)
    if net.readout == "mean":
        return z.mean(0) * 10, (s1, s2)
    y = torch.zeros_like(z[0])
    ys = []
    for t in range(z.shape[0]):
        y = net.beta * y + z[t]
        ys.append(y)
    return torch.stack(ys).mean(0), (s1, s2)


@pytest.mark.parametrize("readout,init,beta", (("mean", "reference", 0.95), ("leaky", "kaiming", 0.9)))
@pytest.mark.parametrize("mode", ("scan", "serial"))
def test_network_matches_torch_reference(cuda, readout, init, beta, mode):
    from hard_resets_compose_b200.shdnet import Net, synthetic_batch
    torch.manual_seed(0)
    net = Net(mode=mode, beta=beta, init=init, readout=readout).to(cuda)
    x, y = synthetic_batch(128, 8, seed=1, device=cuda)
    # scale the first layer so the raster drives spikes in both layers
    with torch.no_grad():
        net.l1.fc.weight.mul_(6.0)
        net.l2.fc.weight.mul_(3.0)
    logits, (s1, s2) = net(x)
    loss = nn.functional.cross_entropy(logits, y)
    grads = torch.autograd.grad(loss, list(net.parameters()))
    rlogits, (r1, r2) = _reference_forward(net, x)
    rloss = nn.functional.cross_entropy(rlogits, y)
    rgrads = torch.autograd.grad(rloss, list(net.parameters()))
    assert s1.sum() > 0 and s2.sum() > 0
    assert torch.equal(s1, r1.detach()) and torch.equal(s2, r2.detach())
    assert rel(logits.detach().cpu().numpy(), rlogits.detach().cpu().numpy()) < 1e-6
    for g, rg in zip(grads, rgrads):
        assert rel(g.cpu().numpy(), rg.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("readout,init,beta,scale", (
    ("mean", "reference", 0.95, (1.0, 1.0)),   # the reference Net as written (lifscan/shdnet.py:53-66)
    ("mean", "reference", 0.95, (6.0, 3.0)),   # the same with both layers driven to spike
    ("leaky", "kaiming", 0.9, (6.0, 3.0)),     # the config-3 benchmark variant
))
def test_network_c3_full_shape(cuda, readout, init, beta, scale):
    """Config 3 at its real shape: B = 64, T = 1024, the 700-channel Bernoulli
    raster of synthetic_batch.  Spikes of both LIF layers (16384 neurons each)
    bit-equal to the plain torch fp32 serial loop on the same GEMM outputs;
    every parameter gradient within 1e-5 relative."""
    from hard_resets_compose_b200.shdnet import Net, synthetic_batch
    torch.manual_seed(1)
    net = Net(mode="scan", beta=beta, init=init, readout=readout).to(cuda)
    x, y = synthetic_batch(1024, 64, seed=2, device=cuda)
    with torch.no_grad():
        net.l1.fc.weight.mul_(scale[0])
        net.l2.fc.weight.mul_(scale[1])
    logits, (s1, s2) = net(x)
    loss = nn.functional.cross_entropy(logits, y)
    grads = torch.autograd.grad(loss, list(net.parameters()))
    rlogits, (r1, r2) = _reference_forward(net, x)
    rloss = nn.functional.cross_entropy(rlogits, y)
    rgrads = torch.autograd.grad(rloss, list(net.parameters()))
    assert s1.sum() > 0
    if scale != (1.0, 1.0):
        assert s2.sum() > 0
    assert torch.equal(s1, r1.detach()) and torch.equal(s2, r2.detach())
    assert rel(logits.detach().cpu().numpy(), rlogits.detach().cpu().numpy()) < 1e-6
    for g, rg in zip(grads, rgrads):
        assert rel(g.cpu().numpy(), rg.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("T,B,din,dout,rate,scale", ((1024, 64, 700, 256, 0.0225, 6.0), (1024, 64, 256, 256, 0.05, 3.0),
                                                   (100, 3, 37, 64, 0.2, 2.0), (257, 5, 1024, 32, 0.01, 10.0)))
def test_spike_producer_matches_linear_then_lif(cuda, T, B, din, dout, rate, scale):
    """The fused spike-input producer (lifb_spike_linear_lif_fwd) against
    nn.Linear then lif_tuned on the same 0/1 raster: S bit-equal (the fused I
    sums in cuBLAS's order), the gradients of x, W and b within 1e-5."""
    from hard_resets_compose_b200 import lifscan as Lm
    from hard_resets_compose_b200.shdnet import spike_linear_lif
    torch.manual_seed(3)
    fc = nn.Linear(din, dout).to(cuda)
    with torch.no_grad():
        fc.weight.mul_(scale)
    x = (torch.rand(T, B, din, device=cuda) < rate).float().requires_grad_(True)
    g = torch.randn(T, B, dout, device=cuda)
    S = spike_linear_lif(x, fc.weight, fc.bias, 0.9)
    gx, gw, gb = torch.autograd.grad(S, (x, fc.weight, fc.bias), g)
    x2 = x.detach().clone().requires_grad_(True)
    I = fc(x2).reshape(T, -1)
    S2 = Lm.lif_tuned(I, torch.zeros(I.shape[1], device=cuda), beta=0.9).reshape(T, B, dout)
    gx2, gw2, gb2 = torch.autograd.grad(S2, (x2, fc.weight, fc.bias), g)
    assert S.sum() > 0
    assert torch.equal(S.view(torch.int32), S2.view(torch.int32))
    for a, r in ((gx, gx2), (gw, gw2), (gb, gb2)):
        assert rel(a.cpu().numpy(), r.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("readout,init,beta", (("mean", "reference", 0.95), ("leaky", "kaiming", 0.9)))
def test_network_c3_spike_producer(cuda, readout, init, beta):
    """Config 3's network with the fused producer in both LIF layers: spikes
    bit-equal to the plain torch fp32 serial restatement, every parameter
    gradient within 1e-5 relative (B = 64, T = 1024)."""
    from hard_resets_compose_b200.shdnet import Net, synthetic_batch
    torch.manual_seed(1)
    net = Net(mode="scan", beta=beta, init=init, readout=readout, producer="spike").to(cuda)
    x, y = synthetic_batch(1024, 64, seed=2, device=cuda)
    with torch.no_grad():
        net.l1.fc.weight.mul_(6.0)
        net.l2.fc.weight.mul_(3.0)
    logits, (s1, s2) = net(x)
    loss = nn.functional.cross_entropy(logits, y)
    grads = torch.autograd.grad(loss, list(net.parameters()))
    rlogits, (r1, r2) = _reference_forward(net, x)
    rloss = nn.functional.cross_entropy(rlogits, y)
    rgrads = torch.autograd.grad(rloss, list(net.parameters()))
    assert s1.sum() > 0 and s2.sum() > 0
    assert torch.equal(s1, r1.detach()) and torch.equal(s2, r2.detach())
    assert rel(logits.detach().cpu().numpy(), rlogits.detach().cpu().numpy()) < 1e-6
    for g, rg in zip(grads, rgrads):
        assert rel(g.cpu().numpy(), rg.cpu().numpy()) < 1e-5


@pytest.mark.parametrize("T,M,beta", ((1024, 1280, 0.9), (1000, 33, 0.99), (17, 5, 0.5), (64, 32, 0.95)))
def test_leaky_integrator_matches_sequential(cuda, T, M, beta):
    """The chunked leaky integrator (lifb_leaky_fwd / lifb_leaky_bwd) against
    the sequential recurrences in fp64: y_t = beta*y_{t-1} + z_t and
    lam_t = g_t + beta*lam_{t+1}, within 1e-6 relative."""
    from hard_resets_compose_b200 import _lib
    from hard_resets_compose_b200._lib import check, ptr, stream_of
    lib = _lib.load()
    g = torch.Generator(device="cpu").manual_seed(T + M)
    z = torch.randn(T, M, generator=g).to(cuda)
    gy = torch.randn(T, M, generator=g).to(cuda)
    Y = torch.empty_like(z)
    lam = torch.empty_like(z)
    check(lib.lifb_leaky_fwd(ptr(z), ptr(Y), T, M, beta, stream_of(z)), "leaky fwd")
    check(lib.lifb_leaky_bwd(ptr(gy), ptr(lam), T, M, beta, stream_of(z)), "leaky bwd")
    torch.cuda.synchronize()
    zd, gd = z.double().cpu(), gy.double().cpu()
    yr = torch.zeros(T, M, dtype=torch.float64)
    lr = torch.zeros(T, M, dtype=torch.float64)
    y = torch.zeros(M, dtype=torch.float64)
    for t in range(T):
        y = beta * y + zd[t]
        yr[t] = y
    l = torch.zeros(M, dtype=torch.float64)
    for t in range(T - 1, -1, -1):
        l = gd[t] + beta * l
        lr[t] = l
    assert float((Y.cpu().double() - yr).abs().max() / yr.abs().max()) < 1e-6
    assert float((lam.cpu().double() - lr).abs().max() / lr.abs().max()) < 1e-6
    # past the one-launch form: refused, so the layer takes the serial path
    assert lib.lifb_leaky_fwd(ptr(z), ptr(Y), 1025, 1, beta, stream_of(z)) == 4
