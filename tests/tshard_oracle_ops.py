"""CPU stand-in for the per-slice phases of the time-sharded scan (test
infrastructure: it drives hard_resets_compose_b200.tshard's host protocol with
the oracle instead of the GPU, so that the protocol runs under gloo on CPU).

Each phase keeps the contract of its lifb_tshard_* counterpart:
  envelope   the slice's envelope map (c, a, b), folded row by row
             (l -> min(u_r, beta*l + x), lifscan/triton_lif.py:698-719)
  slice_map  one map of the whole slice in the [4 + 2*K3, N] layout, from the
             oracle's three-level composition with a single group
             (lifscan/triton_lif.py:828-899), pruned with the entry bound; in
             mode "corrupt" a constant map (a deliberately wrong guess)
  apply      entry = u0 through the earlier maps, then the serial recurrence
  spec_begin the guess of the slice's final state: its last rows run from u_r
  spec_finish the serial recurrence from the (guessed) entry
  repair     the serial recurrence from the new entry; changed = end moved
  bwd        the serial adjoint with lam = 0 above the slice, and (q, p)
  bwd_fix    the serial adjoint with lam_top entering from above
"""
import numpy as np
import torch

from oracle import oracle as O


def _i32(a):
    return np.asarray(a, np.float32).view(np.int32)


def eval_map(mp, u, K3):
    """u through one packed slice map (lifb_tshard_apply's rule): the first
    descending breakpoint x_k <= u selects constant c_k, none selects A*u+B."""
    A, B = mp[0], mp[1]
    cnt = _i32(mp[2])
    X, Cc = mp[4:4 + K3], mp[4 + K3:4 + 2 * K3]
    out = (A * u + B).astype(np.float32)
    done = np.zeros(u.shape, bool)
    for k in range(K3):
        hit = (~done) & (k < cnt) & (X[k] <= u)
        out = np.where(hit, Cc[k], out)
        done |= hit | (k >= cnt)
    return out.astype(np.float32)


class OracleSliceOps:
    def __init__(self, T, N, beta, theta, u_r, alpha=4.0, C=64, K=16, K3=32, mode="maps"):
        self.T, self.N, self.C, self.K, self.K3 = T, N, C, K, K3
        self.beta, self.theta, self.u_r, self.alpha = (np.float32(v) for v in (beta, theta, u_r, alpha))
        self.mode = mode
        self.map_rows = 4 + 2 * K3

    def envelope(self, I):
        x = I.numpy()
        c = np.full(self.N, np.inf, np.float32)
        a = np.ones(self.N, np.float32)
        b = np.zeros(self.N, np.float32)
        for t in range(self.T):
            c = np.minimum(self.u_r, self.beta * c + x[t])
            a = self.beta * a
            b = self.beta * b + x[t]
        return torch.from_numpy(np.stack([c, a, b]))

    def slice_map(self, I, envs, rank, u0):
        e = envs.numpy()
        lo = u0.numpy().copy()
        for q in range(rank):
            lo = np.minimum(e[q, 0], e[q, 1] * lo + e[q, 2]).astype(np.float32)
        m = np.zeros((self.map_rows, self.N), np.float32)
        if self.mode == "corrupt":
            m[1] = 0.5  # A = 0, B = 0.5, no breakpoints: every entry guessed as 0.5
            return torch.from_numpy(m)
        M = self.T // self.C
        _, _, _, d = O.scan_forward_v4(I.numpy(), float(self.beta), float(self.theta), float(self.u_r), lo,
                                       C=self.C, G=M, K=self.K, K2=self.K3, return_internals=True)
        m[0], m[1] = d["SA"][0], d["SB"][0]
        m[2], m[3] = d["SN"][0].view(np.float32), d["SOVF"][0].view(np.float32)
        m[4:4 + self.K3] = d["SX"][0]
        m[4 + self.K3:] = d["SC"][0]
        return torch.from_numpy(m)

    def apply(self, I, maps, rank, u0):
        mp = maps.numpy()
        u = u0.numpy().astype(np.float32).copy()
        for q in range(rank):
            u = eval_map(mp[q], u, self.K3)
        U, S = O.serial_forward(I.numpy(), float(self.beta), float(self.theta), float(self.u_r), u)
        return (torch.from_numpy(u), torch.from_numpy(U), torch.from_numpy(S), torch.from_numpy(U[-1].copy()))

    def tail_segment(self, L=64, W=48):
        """(L, W) of the tail/head forward (lifb_tshard_fwd_tail/_head), or
        None for slices of fewer than two segments."""
        if self.mode == "no_tail" or self.T % L or self.T // L < 2:
            return None
        return L, W

    def fwd_tail(self, I):
        """Segments 1.. from W-row lead-ins from u_r; returns (U, S, guess of
        the slice's final state = the last segment's end)."""
        L, W = self.tail_segment()
        x = I.numpy()
        U = np.zeros_like(x)
        S = np.zeros_like(x)
        b, th, ur = float(self.beta), float(self.theta), float(self.u_r)
        for sg in range(1, self.T // L):
            t0 = max(sg * L - W, 0)
            u = np.full(self.N, self.u_r, np.float32)
            if t0 < sg * L:
                Ul, _ = O.serial_forward(x[t0:sg * L], b, th, ur, u)
                u = Ul[-1].copy()
            Us, Ss = O.serial_forward(x[sg * L:(sg + 1) * L], b, th, ur, u)
            U[sg * L:(sg + 1) * L], S[sg * L:(sg + 1) * L] = Us, Ss
        return torch.from_numpy(U), torch.from_numpy(S), torch.from_numpy(U[-1].copy())

    def fwd_head(self, I, entry, U, S):
        """Segment 0 from entry and the fix-up: U, S exact for entry."""
        U2, S2 = O.serial_forward(I.numpy(), float(self.beta), float(self.theta), float(self.u_r), entry.numpy())
        U.numpy()[:] = U2
        S.numpy()[:] = S2
        return torch.from_numpy(U2[-1].copy())

    def spec_begin(self, I, lead=256):
        x = I.numpy()[-min(lead, self.T):]
        Ug, _ = O.serial_forward(x, float(self.beta), float(self.theta), float(self.u_r),
                                 np.full(self.N, self.u_r, np.float32))
        return torch.from_numpy(Ug[-1].copy())

    def spec_finish(self, I, entry):
        U, S = O.serial_forward(I.numpy(), float(self.beta), float(self.theta), float(self.u_r), entry.numpy())
        return torch.from_numpy(U), torch.from_numpy(S)

    def repair(self, I, entry, U, S, end):
        U2, S2 = O.serial_forward(I.numpy(), float(self.beta), float(self.theta), float(self.u_r), entry.numpy())
        moved = (U2[-1].view(np.uint32) != end.numpy().view(np.uint32)) | (S2[-1] != S.numpy()[-1])
        U.numpy()[:] = U2
        S.numpy()[:] = S2
        end.numpy()[:] = U2[-1]
        return torch.from_numpy(moved.astype(np.int32))

    def _adjoint(self, I, u_prev, U, GS, top):
        _, S = O.serial_forward(I.numpy(), float(self.beta), float(self.theta), float(self.u_r), u_prev.numpy())
        GU = np.zeros_like(S)
        if top is not None:
            # lam_{T-1} = c + beta*J*top: the same as an upstream gradient beta*top on U's last row
            GU[-1] = self.beta * top.numpy()
        Lam = O.serial_backward(I.numpy(), u_prev.numpy(), U.numpy(), S, GS.numpy(), GU, float(self.beta),
                                float(self.theta), float(self.u_r), float(self.alpha), True)
        return Lam, S

    def bwd(self, I, u_prev, U, GS):
        Lam, S = self._adjoint(I, u_prev, U, GS, None)
        p = np.ones(self.N, np.float32)
        for t in range(self.T):
            p = p * (self.beta * (np.float32(1.0) - S[t]))
        return torch.from_numpy(Lam), torch.from_numpy(np.stack([Lam[0], p]))

    def bwd_fix(self, I, u_prev, U, GS, lam_top, Lam):
        L2, _ = self._adjoint(I, u_prev, U, GS, lam_top)
        Lam.numpy()[:] = L2
        return Lam
