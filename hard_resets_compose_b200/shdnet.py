"""Feed-forward hard-reset LIF network 700-256-256-20 on the B200 scan
(the consumer of the hot path, lifscan/shdnet.py:30-66).

`Net` keeps the reference's semantics (lifscan/shdnet.py:53-66): two
`LIFLayer`s (Linear -> lif_tuned on [T, B*H]) and a Linear readout averaged
over time and scaled by 10; LIF weights drawn from U(+-1.5/sqrt(din))
(:34); default beta 0.95 (:54).  Options reproduce the benchmark network
described for config 3 instead: `init="kaiming"` (PyTorch's default
Kaiming-uniform Linear init) and `readout="leaky"` (a non-spiking leaky
integrator y_t = beta*y_{t-1} + W s_t averaged over time), which runs on the
same kernels: the serial forward with theta = +inf never spikes, and its
adjoint with the upstream gradient on U is the integrator's backward.

The SHD data loader of the reference (h5py, :12-27) is not part of this
package; inputs are dense [T, B, 700] spike rasters.
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import lifscan as L


class LIFLayer(nn.Module):
    """Linear(din, dout) then a hard-reset LIF over time (lifscan/shdnet.py:30-50)."""

    def __init__(self, din, dout, beta, mode="scan", K=16, repair=10 ** 6, init="reference"):
        super().__init__()
        self.fc = nn.Linear(din, dout)
        if init == "reference":
            nn.init.uniform_(self.fc.weight, -1.5 / din ** 0.5, 1.5 / din ** 0.5)
        elif init != "kaiming":
            raise ValueError(f"unknown init {init!r}")
        self.beta, self.mode, self.K, self.repair = beta, mode, K, repair

    def forward(self, x):
        Tn, B, _ = x.shape
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
    """y_t = beta*y_{t-1} + z_t, y_0 = 0, over [T, M]: the serial forward with
    theta = +inf (no spike can occur) and its adjoint with the upstream
    gradient on the state (lam_t = g_t + beta*lam_{t+1})."""

    @staticmethod
    def forward(ctx, z, beta):
        z = z.contiguous()
        y0 = torch.zeros(z.shape[1], device=z.device)
        Y, _ = L.serial_forward(z, beta, math.inf, 0.0, y0)
        ctx.save_for_backward(z, y0, Y)
        ctx.beta = beta
        return Y

    @staticmethod
    def backward(ctx, gY):
        z, y0, Y = ctx.saved_tensors
        zeros = torch.zeros_like(Y)  # no gradient reaches the (absent) spikes
        lam = L.serial_backward(z, y0, Y, None, zeros, gY.contiguous(), ctx.beta, math.inf, 0.0, 4.0, True)
        return lam, None


class Net(nn.Module):
    """700-H-H-n_out network (lifscan/shdnet.py:53-66)."""

    def __init__(self, mode="scan", beta=0.95, H=256, n_out=20, din=700, init="reference", readout="mean"):
        super().__init__()
        self.l1 = LIFLayer(din, H, beta, mode, init=init)
        self.l2 = LIFLayer(H, H, beta, mode, init=init)
        self.out = nn.Linear(H, n_out)
        if readout not in ("mean", "leaky"):
            raise ValueError(f"unknown readout {readout!r}")
        self.readout, self.beta = readout, beta

    def set_mode(self, mode):
        self.l1.mode = self.l2.mode = mode

    def forward(self, x):
        s1 = self.l1(x)
        s2 = self.l2(s1)
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
