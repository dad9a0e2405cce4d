"""Feed-forward hard-reset LIF network 700-256-256-20 on the B200 scan
(the consumer of the hot path, lifscan/shdnet.py:30-66).

`Net` keeps the reference's semantics (lifscan/shdnet.py:53-66): two
`LIFLayer`s (Linear -> lif_tuned on [T, B*H]) and a Linear readout averaged
over time and scaled by 10; LIF weights drawn from U(+-1.5/sqrt(din))
(:34); default beta 0.95 (:54).  Options reproduce the benchmark network
described for config 3 instead: `init="kaiming"` (PyTorch's default
Kaiming-uniform Linear init) and `readout="leaky"` (a non-spiking leaky
integrator y_t = beta*y_{t-1} + W s_t averaged over time), a linear
recurrence run as 64-row chunks with one carried value each
(lifb_leaky_fwd / lifb_leaky_bwd).

`producer="spike"` runs each LIF layer's Linear and recurrence as one fused
kernel (lifb_spike_linear_lif_fwd) for spike inputs: the input is read as a
bitmask of its active elements (lifb_spike_mask; a fused layer hands the mask
of its own spikes to the next one), I is never written to memory, and each
of its elements sums the active inputs' weights in the order cuBLAS's fp32
GEMM does, so the spikes are the same bits as with `producer="linear"`
(nn.Linear, then lif_tuned).  The backward is lif_tuned's adjoint from V,
then the weight and bias gradients over the active inputs only
(lifb_spike_linear_wgrad) and dI W for the input's gradient.  The readout
Linear then keeps torch's forward and takes the same sparse weight gradient
from layer 2's spike mask (`spike_input_linear`).

The SHD data loader of the reference (h5py, :12-27) is not part of this
package; inputs are dense [T, B, 700] spike rasters.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import _lib
from . import lifscan as L
from ._lib import check, ptr, stream_of


_MASK_ATTR = "_lifb_spike_mask"


def spike_mask(x2d):
    """Spike mask [R, lifb_spike_mask_stride(D)] int32 of a [R, D] fp32 tensor
    (lifb_spike_mask): bit q of word k set where element 32k + q is nonzero,
    word ceil(D/32) bit 0 set on rows with a nonzero value other than 1."""
    R, D = x2d.shape
    lib = _lib.load()
    m = torch.empty(R, lib.lifb_spike_mask_stride(D), dtype=torch.int32, device=x2d.device)
    with torch.cuda.device(x2d.device):
        check(lib.lifb_spike_mask(ptr(x2d), ptr(m), R, D, stream_of(x2d)), "spike_mask")
    return m


def _carried_mask(x):
    """The mask a fused layer attached to its spike output x, if x is still
    that tensor, unmodified; else None."""
    rec = getattr(x, _MASK_ATTR, None)
    if rec is None:
        return None
    m, version = rec
    return m if version == x._version else None


class SpikeLinearLIF(torch.autograd.Function):
    """Linear on a spike input then lif_tuned's hard-reset LIF (theta, u_r,
    sigmoid surrogate alpha, detached reset), forward fused in one kernel
    (lifb_spike_linear_lif_fwd).  Returns S [T, B, Dout] and the spike mask
    of S (not differentiable).  The backward is lif_tuned's adjoint from V,
    then the weight and bias gradients over the input's active elements
    (lifb_spike_linear_wgrad) and, when needed, dI W for the input."""

    @staticmethod
    def forward(ctx, x, xmask, weight, bias, beta, theta, u_r, alpha, mode):
        x = x.contiguous()
        T, B, din = x.shape
        dout = weight.shape[0]
        lib = _lib.load()
        if xmask is None:
            xmask = spike_mask(x.view(T * B, din))
        V = torch.empty(T, B * dout, device=x.device)
        S = torch.empty(T, B, dout, device=x.device)
        smask = torch.empty(T * B, lib.lifb_spike_mask_stride(dout), dtype=torch.int32, device=x.device)
        with torch.cuda.device(x.device):
            check(lib.lifb_spike_linear_lif_fwd(ptr(x), ptr(xmask), ptr(weight.contiguous()),
                                                ptr(None if bias is None else bias.contiguous()), None, ptr(V),
                                                ptr(S), ptr(smask), T, B, din, dout, float(beta), float(theta),
                                                float(u_r), stream_of(x)), "spike_linear_lif")
        ctx.save_for_backward(x, xmask, weight, V)
        ctx.cfg = (beta, theta, alpha, mode, bias is not None)
        ctx.mark_non_differentiable(smask)
        return S, smask

    @staticmethod
    def backward(ctx, gS, _gmask):
        x, xmask, weight, V = ctx.saved_tensors
        beta, theta, alpha, mode, has_bias = ctx.cfg
        T, N = V.shape
        B, din, dout = x.shape[1], x.shape[2], weight.shape[0]
        # lif_tuned's backward for this shape (its forward is the single pass)
        lam = L.lif_backward_v(V, gS.reshape(T, N), beta, theta, alpha,
                               C=T if mode == "serial" else L.scan_chunk_bwd(T, N))
        dI = lam.reshape(T * B, dout)
        gx = dense_dgrad(dI, weight).reshape(T, B, din) if ctx.needs_input_grad[0] else None
        gw, gb = _spike_wgrad(dI, x, xmask, ctx.needs_input_grad[2], has_bias and ctx.needs_input_grad[3])
        _lib.poll_device("spike_linear_lif")
        return gx, None, gw, gb, None, None, None, None, None


def dense_dgrad_applies(din, dout):
    """Whether lifb_dense_dgrad takes a layer of this shape."""
    return dout % 4 == 0 and din in (64, 128, 256)


def dense_dgrad(dY, weight):
    """dY [R, Dout] . weight [Dout, Din], a Linear layer's input gradient: on
    the tensor cores (lifb_dense_dgrad, three TF32 products accumulated in
    fp32, within about 1e-6..4e-6 relative of an fp32 GEMM) where the shape
    allows, else torch's fp32 GEMM."""
    dY = dY.contiguous()
    weight = weight.contiguous()
    R, dout = dY.shape
    din = weight.shape[1]
    if not dense_dgrad_applies(din, dout):
        return dY.mm(weight)
    lib = _lib.load()
    dX = torch.empty(R, din, device=dY.device)
    nb = lib.lifb_dense_dgrad_workspace_bytes(din, dout)
    ws = torch.empty(nb, dtype=torch.uint8, device=dY.device)
    with torch.cuda.device(dY.device):
        check(lib.lifb_dense_dgrad(ptr(dY), ptr(weight), ptr(dX), R, din, dout, ptr(ws), nb, stream_of(dY)),
              "dense_dgrad")
    return dX


def _spike_wgrad(dI, x, xmask, want_w, want_b):
    """Weight and bias gradients dI^T x and dI.sum(0) of a Linear layer whose
    input x [..., Din] has the spike mask xmask, over x's active elements only
    (lifb_spike_linear_wgrad); (None, None) parts that are not wanted."""
    if not (want_w or want_b):
        return None, None
    R, dout = dI.shape
    din = x.shape[-1]
    lib = _lib.load()
    gw = torch.empty(dout, din, device=x.device)
    gb = torch.empty(dout, device=x.device) if want_b else None
    ws = torch.empty(max(lib.lifb_spike_linear_wgrad_workspace_bytes(R, din, dout), 1), dtype=torch.uint8,
                     device=x.device)
    with torch.cuda.device(x.device):
        check(lib.lifb_spike_linear_wgrad(ptr(dI), ptr(x), ptr(xmask), ptr(gw), ptr(gb), R, din, dout, ptr(ws),
                                          ws.numel(), stream_of(x)), "spike_linear_wgrad")
    return (gw if want_w else None), gb


class SpikeInputLinear(torch.autograd.Function):
    """torch.nn.Linear on a spike input x [..., Din] with mask xmask: the
    forward is torch's linear itself (the same bits as nn.Linear); the
    backward computes dX = dY W as torch does and the weight and bias
    gradients over x's active elements only (lifb_spike_linear_wgrad)."""

    @staticmethod
    def forward(ctx, x, xmask, weight, bias):
        y = nn.functional.linear(x, weight, bias)
        ctx.save_for_backward(x, xmask, weight)
        ctx.has_bias = bias is not None
        return y

    @staticmethod
    def backward(ctx, gy):
        x, xmask, weight = ctx.saved_tensors
        g2 = gy.reshape(-1, weight.shape[0]).contiguous()
        gx = dense_dgrad(g2, weight).reshape(x.shape) if ctx.needs_input_grad[0] else None
        gw, gb = _spike_wgrad(g2, x, xmask, ctx.needs_input_grad[2], ctx.has_bias and ctx.needs_input_grad[3])
        _lib.poll_device("spike_input_linear")
        return gx, None, gw, gb


def spike_input_linear(x, weight, bias=None):
    """nn.functional.linear(x, weight, bias) for a spike input x [..., Din]
    (Din <= 1024, Dout % 4 == 0), with the sparse weight gradient; x's carried
    spike mask is used when it has one."""
    x = x.contiguous()
    m = _carried_mask(x)
    if m is None:
        m = spike_mask(x.reshape(-1, x.shape[-1]))
    return SpikeInputLinear.apply(x, m, weight, bias)


def spike_linear_lif(x, weight, bias, beta, theta=1.0, u_r=0.0, alpha=4.0, mode="scan"):
    """S = lif_tuned(linear(x, weight, bias).reshape(T, -1), 0, ...) for a
    spike input x [T, B, Din], forward fused (SpikeLinearLIF).  S carries
    its spike mask to a fused layer that consumes it."""
    S, m = SpikeLinearLIF.apply(x, _carried_mask(x), weight, bias, beta, theta, u_r, alpha, mode)
    setattr(S, _MASK_ATTR, (m, S._version))
    return S


def spike_producer_applies(din, dout):
    """True when the fused producer serves a Linear(din, dout) layer."""
    return 0 < din <= 1024 and dout % 32 == 0


class LIFLayer(nn.Module):
    """Linear(din, dout) then a hard-reset LIF over time (lifscan/shdnet.py:30-50).
    producer="spike": the fused spike-input producer (the input must hold
    0/1 spikes), where it applies; "linear": nn.Linear then lif_tuned."""

    def __init__(self, din, dout, beta, mode="scan", K=16, repair=10 ** 6, init="reference", producer="linear"):
        super().__init__()
        self.fc = nn.Linear(din, dout)
        if init == "reference":
            nn.init.uniform_(self.fc.weight, -1.5 / din ** 0.5, 1.5 / din ** 0.5)
        elif init != "kaiming":
            raise ValueError(f"unknown init {init!r}")
        if producer not in ("linear", "spike"):
            raise ValueError(f"unknown producer {producer!r}")
        self.beta, self.mode, self.K, self.repair, self.producer = beta, mode, K, repair, producer

    def forward(self, x):
        Tn, B, _ = x.shape
        if (self.producer == "spike" and self.mode in ("scan", "serial") and x.is_cuda
                and spike_producer_applies(self.fc.in_features, self.fc.out_features)):
            return spike_linear_lif(x, self.fc.weight, self.fc.bias, self.beta, 1.0, 0.0, 4.0, self.mode)
        I = self.fc(x).reshape(Tn, -1).contiguous()
        u0 = torch.zeros(I.shape[1], device=I.device)
        if self.mode == "auto":
            s = L.lif_auto(I, u0, beta=self.beta, theta=1.0, u_r=0.0, alpha=4.0, K=self.K, repair=0)
        elif self.mode in ("serial", "scan"):
            s = L.lif_tuned(I, u0, beta=self.beta, theta=1.0, u_r=0.0, alpha=4.0, mode=self.mode, K=self.K,
                            repair=self.repair)
        else:
            raise ValueError(f"unknown mode {self.mode!r}")
        return s.reshape(Tn, B, -1)


class _LeakyIntegrator(torch.autograd.Function):
    """y_t = beta*y_{t-1} + z_t, y_0 = 0, over [T, M], and its adjoint
    lam_t = g_t + beta*lam_{t+1}: the chunked linear recurrences of
    lifb_leaky_fwd / lifb_leaky_bwd (T <= 1024), else the serial forward with
    theta = +inf (no spike can occur) and its adjoint with the upstream
    gradient on the state."""

    @staticmethod
    def forward(ctx, z, beta):
        z = z.contiguous()
        T, M = z.shape
        lib = _lib.load()
        ctx.beta = beta
        if T <= 1024:
            Y = torch.empty_like(z)
            with torch.cuda.device(z.device):
                check(lib.lifb_leaky_fwd(ptr(z), ptr(Y), T, M, float(beta), stream_of(z)), "leaky integrator")
            ctx.chunked = True
            return Y
        y0 = torch.zeros(M, device=z.device)
        Y, _ = L.serial_forward(z, beta, math.inf, 0.0, y0)
        ctx.save_for_backward(z, y0, Y)
        ctx.chunked = False
        return Y

    @staticmethod
    def backward(ctx, gY):
        gY = gY.contiguous()
        if ctx.chunked:
            T, M = gY.shape
            lam = torch.empty_like(gY)
            with torch.cuda.device(gY.device):
                check(_lib.load().lifb_leaky_bwd(ptr(gY), ptr(lam), T, M, float(ctx.beta), stream_of(gY)),
                      "leaky integrator adjoint")
            return lam, None
        z, y0, Y = ctx.saved_tensors
        zeros = torch.zeros_like(Y)  # no gradient reaches the (absent) spikes
        lam = L.serial_backward(z, y0, Y, None, zeros, gY, ctx.beta, math.inf, 0.0, 4.0, True)
        return lam, None


class Net(nn.Module):
    """700-H-H-n_out network (lifscan/shdnet.py:53-66)."""

    def __init__(self, mode="scan", beta=0.95, H=256, n_out=20, din=700, init="reference", readout="mean",
                 producer="linear"):
        super().__init__()
        self.l1 = LIFLayer(din, H, beta, mode, init=init, producer=producer)
        self.l2 = LIFLayer(H, H, beta, mode, init=init, producer=producer)
        self.out = nn.Linear(H, n_out)
        if readout not in ("mean", "leaky"):
            raise ValueError(f"unknown readout {readout!r}")
        self.readout, self.beta = readout, beta

    def set_mode(self, mode):
        self.l1.mode = self.l2.mode = mode

    def forward(self, x):
        s1 = self.l1(x)
        s2 = self.l2(s1)
        if (self.l2.producer == "spike" and s2.is_cuda and self.out.in_features <= 1024
                and self.out.out_features % 4 == 0):
            z = spike_input_linear(s2, self.out.weight, self.out.bias)  # nn.Linear's bits, sparse dW
        else:
            z = self.out(s2)  # [T, B, n_out]
        if self.readout == "mean":
            return z.mean(0) * 10, (s1, s2)
        Tn, B, C = z.shape
        y = _LeakyIntegrator.apply(z.reshape(Tn, B * C), self.beta).reshape(Tn, B, C)
        return y.mean(0), (s1, s2)


def synthetic_batch(T, B, channels=700, seed=0, device="cuda"):
    """Bernoulli spike raster x[t, b, c] = rand < r_c with r_c ~ U(0.005, 0.04)
    per channel, and labels ~ randint(0, 20) (the config-3 benchmark input)."""
    g = torch.Generator().manual_seed(seed)
    rate = 0.005 + 0.035 * torch.rand(channels, generator=g)
    x = (torch.rand(T, B, channels, generator=g) < rate).float()
    y = torch.randint(0, 20, (B,), generator=g)
    return x.to(device), y.to(device)
