"""Time-sharded exact LIF scan: one slice of the time axis per GPU.

The reference scans a whole sequence on one device (scan_forward_v4,
lifscan/triton_lif.py:944-983; scan_backward_tiled, :512-526).  Here rank r
of a process group owns rows [r*T, (r+1)*T) of a [P*T, N] sequence and the
ranks exchange only small per-neuron summaries with all-gathers:

forward (entry_mode "maps"; "speculate" replaces steps 1-3, see tshard_forward)
  1. envelope   each slice's envelope map l -> min(c, a*l + b)        3 floats
  2. slice map  each slice composed into one pruned piecewise map,
                pruned with the entry bound folded from the envelopes   4 + 2*K3 floats
  3. apply      entry = u0 through the earlier slices' maps; super carry,
                replay and local fix-up from that entry
  4. repair     all-gather of slice end states; a slice whose entry
                changed replays until its rows rejoin; until no end moves
backward
  5. adjoint    each slice from lam = 0 above it, summarised as
                lam_0 = q + p * lam_above                               2 floats
  6. fix        lam above each slice folded from the later slices' (q, p);
                the rows above each chunk's last spike are redone

U and S equal the serial fp32 recurrence over all P*T rows bit for bit (an
overflowed slice map only makes step 3 a guess that step 4 corrects); the
gradients equal its adjoint within rounding.

The collective calls go through a `comm` object (all_gather of a tensor from
every rank, in rank order), and the per-slice phases through an `ops` object;
`CudaSliceOps` runs them on this GPU through liblifb.so.  Every rank takes
the same collective steps in the same order.
"""
from __future__ import annotations

import threading

import torch
import torch.distributed as dist

from . import _lib
from ._lib import check, ptr, stream_of

__all__ = ["TorchComm", "LocalComm", "run_local", "CudaSliceOps", "tshard_forward", "tshard_backward", "LIFTimeSharded", "lif_tshard",
           "slice_rows"]


def slice_rows(T_total, world, rank):
    """Rows [start, stop) of rank `rank` when T_total rows are split evenly."""
    if T_total % world:
        raise ValueError(f"T={T_total} does not split evenly over {world} ranks")
    T = T_total // world
    return rank * T, (rank + 1) * T


class TorchComm:
    """all_gather over a torch.distributed process group (NCCL on GPUs, gloo on CPU)."""

    def __init__(self, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def shift(self, t):
        """t of rank r-1 on rank r (rank 0 receives None); every rank sends
        its t to rank r+1."""
        t = t.contiguous()
        ops = []
        if self.rank + 1 < self.world:
            ops.append(dist.P2POp(dist.isend, t, self.rank + 1, group=self.group))
        buf = None
        if self.rank > 0:
            buf = torch.empty_like(t)
            ops.append(dist.P2POp(dist.irecv, buf, self.rank - 1, group=self.group))
        if ops:
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        return buf

    def all_gather(self, t):
        t = t.contiguous()
        if t.is_cuda:
            out = torch.empty((self.world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
            dist.all_gather_into_tensor(out, t, group=self.group)
            return out
        parts = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(parts, t, group=self.group)
        return torch.stack(parts)


class LocalComm:
    """Ranks emulated as threads of one process (one GPU or the CPU): rank r
    is the r-th thread, all_gather meets the others at a barrier.  Build one
    with LocalComm.group(world) and hand comm r to thread r."""

    class _Shared:
        def __init__(self, world, timeout):
            self.slots = [None] * world
            self.barrier = threading.Barrier(world, timeout=timeout)

    def __init__(self, shared, world, rank):
        self.shared, self.world, self.rank = shared, world, rank

    @classmethod
    def group(cls, world, timeout=60.0):
        sh = cls._Shared(world, timeout)
        return [cls(sh, world, r) for r in range(world)]

    def all_gather(self, t):
        sh = self.shared
        sh.slots[self.rank] = t.contiguous()
        sh.barrier.wait()
        out = torch.stack(sh.slots)
        sh.barrier.wait()  # every rank has its copy before the slots are reused
        return out

    def shift(self, t):
        g = self.all_gather(t)
        return g[self.rank - 1].clone() if self.rank > 0 else None


def run_local(world, fn):
    """Runs fn(comm) for every emulated rank in its own thread and returns the
    results in rank order; the first exception of any rank is raised (the
    barrier is broken so that the other ranks stop too)."""
    comms = LocalComm.group(world)
    out, errs = [None] * world, [None] * world

    def body(r):
        try:
            out[r] = fn(comms[r])
        except BaseException as e:  # noqa: BLE001 - re-raised below
            errs[r] = e
            comms[r].shared.barrier.abort()

    th = [threading.Thread(target=body, args=(r,)) for r in range(world)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    for e in errs:
        if e is not None and not isinstance(e, threading.BrokenBarrierError):
            raise e
    for e in errs:
        if e is not None:
            raise e
    return out


class CudaSliceOps:
    """The per-slice phases on this GPU (include/lifscan_b200.h, lifb_tshard_*)."""

    def __init__(self, T, N, device, beta, theta, u_r, alpha=4.0, C=64, G=16, K=16, K2=32, K3=64, C_bwd=4096):
        if T % (C * G):
            raise ValueError(f"slice length {T} is not a multiple of C*G = {C * G}")
        while T % C_bwd:
            C_bwd //= 2
        self.T, self.N, self.dev = T, N, torch.device(device)
        self.beta, self.theta, self.u_r, self.alpha = float(beta), float(theta), float(u_r), float(alpha)
        self.C, self.G, self.K, self.K2, self.K3, self.Cb = C, G, K, K2, K3, C_bwd
        L = self.L = _lib.load()
        self._nb = L.lifb_tshard_workspace_bytes(T, N, C, G, K, K2)
        nbb = L.lifb_tshard_bwd_workspace_bytes(T, N, C_bwd)
        if self._nb == 0 or nbb == 0:
            raise ValueError("time-sharded scan: invalid slice shape")
        self.ws = None  # scratch of entry mode "maps", allocated on first use
        self.wsb = torch.empty(nbb, dtype=torch.uint8, device=self.dev)
        self.map_rows = 4 + 2 * K3

    def _ws(self):
        if self.ws is None:
            self.ws = torch.empty(self._nb, dtype=torch.uint8, device=self.dev)
        return ptr(self.ws), self.ws.numel()

    def envelope(self, I):
        env = torch.empty(3, self.N, device=self.dev)
        with torch.cuda.device(self.dev):
            check(self.L.lifb_tshard_envelope(ptr(I), self.T, self.N, self.C, self.G, self.K, self.K2, self.beta,
                                              self.u_r, ptr(env), *self._ws(), stream_of(I)), "tshard envelope")
        return env

    def slice_map(self, I, envs, rank, u0):
        m = torch.empty(self.map_rows, self.N, device=self.dev)
        with torch.cuda.device(self.dev):
            check(self.L.lifb_tshard_slice_map(ptr(I), ptr(envs), rank, ptr(u0), self.T, self.N, self.beta,
                                               self.theta, self.u_r, self.C, self.G, self.K, self.K2, self.K3,
                                               ptr(m), *self._ws(), stream_of(I)), "tshard slice map")
        return m

    def apply(self, I, maps, rank, u0):
        entry = torch.empty(self.N, device=self.dev)
        end = torch.empty(self.N, device=self.dev)
        U = torch.empty_like(I)
        S = torch.empty_like(I)
        with torch.cuda.device(self.dev):
            check(self.L.lifb_tshard_apply(ptr(I), ptr(maps), rank, self.K3, ptr(u0), ptr(entry), ptr(U), ptr(S),
                                           ptr(end), self.T, self.N, self.beta, self.theta, self.u_r, self.C,
                                           self.G, self.K, self.K2, *self._ws(), stream_of(I)), "tshard apply")
        return entry, U, S, end

    # Segments of a slice's replay in entry mode "speculate": the first
    # segment is replayed alone once the entry has arrived (one chain of L
    # rows on the step's critical path), the others at once from their
    # lead-ins before that, so L is short: 4096 rows, with 4096-row lead-ins
    # (config 4's trajectories merge within ~2100 rows at p99).
    TAIL_L = 4096

    def tail_segment(self):
        """(L, W) of the tail/head forward of this slice, or None when the
        slice has fewer than two segments (then the lead-in pass is used)."""
        from .lifscan import SPEC_LEAD
        L = self.TAIL_L
        if self.T % L or self.T // L < 2 or self.N % 4:
            return None
        return L, SPEC_LEAD

    def fwd_tail(self, I):
        """U, S of segments 1.. of the slice from their fused lead-ins, and the
        guess of the slice's final state (lifb_tshard_fwd_tail)."""
        L, W = self.tail_segment()
        ws = self._tail_ws(L)
        U = torch.empty_like(I)
        S = torch.empty_like(I)
        g = torch.empty(self.N, device=self.dev)
        with torch.cuda.device(self.dev):
            check(self.L.lifb_tshard_fwd_tail(ptr(I), ptr(U), ptr(S), self.T, self.N, self.beta, self.theta, self.u_r,
                                              L, W, ptr(g), ptr(ws), ws.numel(), stream_of(I)),
                  "tshard forward (tail)")
        return U, S, g

    def fwd_head(self, I, entry, U, S):
        """Segment 0 from `entry` and the fix-up of the slice
        (lifb_tshard_fwd_head): U, S exact for entry; returns the end state."""
        L, _ = self.tail_segment()
        ws = self._tail_ws(L)
        end = torch.empty(self.N, device=self.dev)
        with torch.cuda.device(self.dev):
            check(self.L.lifb_tshard_fwd_head(ptr(I), ptr(entry), ptr(U), ptr(S), ptr(end), self.T, self.N, self.beta,
                                              self.theta, self.u_r, L, ptr(ws), ws.numel(), stream_of(I)),
                  "tshard forward (head)")
        return end

    def _tail_ws(self, L):
        if getattr(self, "_tws", None) is None:
            nb = self.L.lifb_scan_fwd_spec_workspace_bytes(self.T, self.N, L)
            self._tws = torch.empty(max(nb, 1), dtype=torch.uint8, device=self.dev)
        return self._tws

    def _spec_ws(self):
        if getattr(self, "_sws", None) is None:
            from .lifscan import SPEC_LEAD, spec_segment
            L, W = spec_segment(self.T, self.N)
            self._sL, self._sW = L, (W if W > 0 else min(SPEC_LEAD, self.T))
            nb = self.L.lifb_scan_fwd_spec_workspace_bytes(self.T, self.N, L)
            self._sws = torch.empty(max(nb, 1), dtype=torch.uint8, device=self.dev)
        return self._sws

    def spec_begin(self, I):
        """Lead-ins of the slice's segments (lifb_scan_fwd_spec_begin) and the
        guess of its final state: its last rows run from u_r."""
        ws = self._spec_ws()
        g = torch.empty(self.N, device=self.dev)
        with torch.cuda.device(self.dev):
            check(self.L.lifb_scan_fwd_spec_begin(ptr(I), self.T, self.N, self.beta, self.theta, self.u_r, self._sL,
                                                  self._sW, ptr(g), ptr(ws), ws.numel(), stream_of(I)),
                  "tshard speculative lead-ins")
        return g

    def spec_finish(self, I, entry):
        """U, S of the slice from `entry` (lifb_scan_fwd_spec_finish, after
        spec_begin): exact for that entry."""
        ws = self._spec_ws()
        U = torch.empty_like(I)
        S = torch.empty_like(I)
        with torch.cuda.device(self.dev):
            check(self.L.lifb_scan_fwd_spec_finish(ptr(I), ptr(entry), ptr(U), ptr(S), self.T, self.N, self.beta,
                                                   self.theta, self.u_r, self._sL, ptr(ws), ws.numel(),
                                                   stream_of(I)), "tshard speculative forward")
        return U, S

    def repair(self, I, entry, U, S, end):
        changed = torch.empty(self.N, dtype=torch.int32, device=self.dev)
        with torch.cuda.device(self.dev):
            check(self.L.lifb_tshard_repair(ptr(I), ptr(entry), ptr(U), ptr(S), ptr(end), ptr(changed), self.T,
                                            self.N, self.beta, self.theta, self.u_r, stream_of(I)), "tshard repair")
        return changed

    def bwd(self, I, u_prev, U, GS):
        Lam = torch.empty_like(I)
        pq = torch.empty(2, self.N, device=self.dev)
        with torch.cuda.device(self.dev):
            check(self.L.lifb_tshard_bwd(ptr(I), ptr(u_prev), ptr(U), ptr(GS), ptr(Lam), ptr(pq), self.T, self.N,
                                         self.beta, self.theta, self.u_r, self.alpha, self.Cb, ptr(self.wsb),
                                         self.wsb.numel(), stream_of(I)), "tshard adjoint")
        return Lam, pq

    def bwd_fix(self, I, u_prev, U, GS, lam_top, Lam):
        with torch.cuda.device(self.dev):
            check(self.L.lifb_tshard_bwd_fix(ptr(I), ptr(u_prev), ptr(U), ptr(GS), ptr(lam_top), ptr(Lam), self.T,
                                             self.N, self.beta, self.theta, self.alpha, self.Cb, ptr(self.wsb),
                                             self.wsb.numel(), stream_of(I)), "tshard adjoint fix-up")
        return Lam


def _mark(timeline, name, ref):
    """Marks the end of a protocol phase: an NVTX marker for profilers (CUDA
    tensors only), and, when timing, (name, CUDA event recorded now on ref's
    stream) appended to the timeline."""
    if ref.is_cuda:
        torch.cuda.nvtx.mark(name)
    if timeline is not None:
        e = torch.cuda.Event(enable_timing=True)
        e.record(torch.cuda.current_stream(ref.device))
        timeline.append((name, e))


def tshard_forward(I, u0, ops, comm, info=None, entry_mode="speculate", timeline=None):
    """Forward of this rank's slice I [T, N] (u0: the state before row 0 of
    the whole sequence, the same on every rank) -> (U, S, entry), where entry
    is the exact state before this slice's first row.

    entry_mode "maps": the entry of every slice comes from the gathered slice
    maps (steps 1-3 of the module docstring), exact unless a map overflowed.
    entry_mode "speculate": every slice runs the lead-ins of its segments and,
    in the same launch, its last few thousand rows from u_r (as if its neuron
    had just spiked), and hands that guess of its final state to the next
    slice (a point-to-point shift of N floats) as that slice's entry; all
    slices then replay at once.  Hard resets make the guess exact in almost
    every neuron, and the repair replays the others from the exact entry only
    until their rows rejoin (no map is built; the envelope and map exchanges
    are skipped).
    Both give the same bits.  `info` (a dict) receives the number of repair
    rounds and the neurons repaired per round; `timeline` (a list, CUDA only)
    receives (phase, CUDA event) pairs marking the end of each phase."""
    R, r = comm.world, comm.rank
    N = I.shape[1]
    if entry_mode == "maps":
        env = ops.envelope(I)
        envs = comm.all_gather(env)
        m = ops.slice_map(I, envs, r, u0)
        maps = comm.all_gather(m)
        entry, U, S, end = ops.apply(I, maps, r, u0)
    elif entry_mode == "speculate" and getattr(ops, "tail_segment", lambda: None)():
        # every segment but the first replays at once from its fused lead-in;
        # the last one's end guesses this slice's final state, which the next
        # slice takes as its entry; then the first segment from the entry and
        # the slice's fix-up
        _mark(timeline, "start", I)
        U, S, guess = ops.fwd_tail(I)
        _mark(timeline, "tail", I)
        entry = comm.shift(guess)
        entry = u0.clone() if r == 0 else entry
        _mark(timeline, "shift", I)
        end = ops.fwd_head(I, entry, U, S)
        _mark(timeline, "head", I)
    elif entry_mode == "speculate":
        # the previous slice's last rows lead the guess (u_r before them) to
        # the exact entry state in all but a few neurons
        _mark(timeline, "start", I)
        guess = ops.spec_begin(I)  # lead-ins, and a guess of this slice's final state
        _mark(timeline, "lead_in", I)
        entry = comm.shift(guess)  # the previous slice's guess is this one's entry
        entry = u0.clone() if r == 0 else entry
        _mark(timeline, "shift", I)
        U, S = ops.spec_finish(I, entry)
        end = U[-1].clone()
        _mark(timeline, "slice", I)
    else:
        raise ValueError(f"unknown entry_mode {entry_mode!r}")
    # cross-slice repair: rank r's rows are exact once slices 0..r-1 are, so
    # R-1 rounds suffice; stop as soon as no slice end moved
    flag = torch.ones(1, dtype=end.dtype, device=end.device)
    rounds, repaired = 0, []
    for it in range(R - 1):
        g = comm.all_gather(torch.cat([end, flag]))
        _mark(timeline, f"gather{it}", I)
        if it == 0:
            need = r > 0  # every slice end is new: no flags to read (no host sync)
        else:
            flags = g[:, N].tolist()
            if I.is_cuda:  # the host has just waited: fold in the device status
                _lib.check_device("time-sharded forward")
            if not any(f != 0.0 for f in flags[:R - 1]):
                break
            need = r > 0 and flags[r - 1] != 0.0
        rounds += 1
        if need:
            entry.copy_(g[r - 1, :N])
            changed = ops.repair(I, entry, U, S, end)
            cnt = changed.sum()
            flag = (cnt > 0).to(end.dtype).reshape(1)
            repaired.append(cnt)
            _mark(timeline, f"repair{it}", I)
        else:
            flag = torch.zeros(1, dtype=end.dtype, device=end.device)
    if info is not None:
        info["repair_rounds"] = rounds
        info["repaired"] = [int(c) for c in repaired]
    return U, S, entry


def tshard_backward(I, entry, U, GS, ops, comm, beta, timeline=None):
    """Adjoint of this rank's slice (entry: the state before its first row,
    from tshard_forward) -> (Lam, du0); du0 = beta * Lam[0] on rank 0, zeros
    on the others (their u0 does not enter their rows)."""
    R, r = comm.world, comm.rank
    _mark(timeline, "bwd_start", I)
    Lam, pq = ops.bwd(I, entry, U, GS)
    _mark(timeline, "adjoint", I)
    g = comm.all_gather(pq)
    _mark(timeline, "gather_pq", I)
    top = torch.zeros_like(entry)
    for q in range(R - 1, r, -1):
        top = torch.addcmul(g[q, 0], g[q, 1], top)  # q + p * lam_above, one launch
    _mark(timeline, "fold", I)
    Lam = ops.bwd_fix(I, entry, U, GS, top, Lam)
    _mark(timeline, "fix", I)
    du0 = Lam[0] * beta if r == 0 else torch.zeros_like(entry)
    return Lam, du0


class LIFTimeSharded(torch.autograd.Function):
    """lif_tuned (lifscan/triton_lif.py:1009-1047: spikes out, sigmoid
    surrogate, detached reset) over a sequence sharded along time."""

    @staticmethod
    def forward(ctx, I, u0, beta, theta, u_r, alpha, ops, comm, entry_mode="speculate"):
        U, S, entry = tshard_forward(I.contiguous(), u0.contiguous(), ops, comm, entry_mode=entry_mode)
        ctx.save_for_backward(I, U, entry)
        ctx.ops, ctx.comm, ctx.beta = ops, comm, float(beta)
        return S

    @staticmethod
    def backward(ctx, gS):
        I, U, entry = ctx.saved_tensors
        dI, du0 = tshard_backward(I, entry, U, gS.contiguous(), ctx.ops, ctx.comm, ctx.beta)
        if I.is_cuda:
            _lib.poll_device("lif_tshard")
        return dI, du0, None, None, None, None, None, None, None


def lif_tshard(I, u0, beta=0.9, theta=1.0, u_r=0.0, alpha=4.0, group=None, C=64, G=16, K=16, K2=32, K3=64,
               ops=None, comm=None, entry_mode="speculate"):
    """Spikes of this rank's time slice I [T, N] of a sequence split evenly
    over the ranks of `group` (rank order = time order).  Differentiable in I
    and u0 like lif_tuned; one process per GPU.  entry_mode: see
    tshard_forward (C, G, K, K2, K3 shape the maps of entry_mode "maps")."""
    if not I.is_cuda and ops is None:
        raise RuntimeError("lif_tshard needs CUDA tensors (this implementation has no CPU path)")
    comm = comm or TorchComm(group)
    ops = ops or CudaSliceOps(I.shape[0], I.shape[1], I.device, beta, theta, u_r, alpha, C, G, K, K2, K3)
    return LIFTimeSharded.apply(I, u0, beta, theta, u_r, alpha, ops, comm, entry_mode)
