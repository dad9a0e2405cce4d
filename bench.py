#!/usr/bin/env python
"""Benchmark of the exact hard-reset LIF scan on B200 (driver contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

Workload (config 2, the one the headline metric is quoted on):
lif_tuned forward+backward, B*N = 16384 neurons per GPU (B = 64 x 256),
T = 1024, x ~ N(0.05, 0.2^2) fp32, beta = 0.99, theta = 1, u_r = 0, u0 = 0,
the default sigmoid surrogate (alpha = 4, detached reset), upstream gradient
on the spikes ~ N(0, 1).  Inputs are drawn on the CPU from a seeded
torch.Generator and copied to the device (synthetic data of the config's
shape and distribution).  A step = one lif_tuned forward + backward
(torch.autograd.backward(S, GS)) through the public API.

Multi-GPU: one process per GPU (torchrun); every rank owns its own batch
shard of 16384 neurons (weak scaling, no data-path collective); the step time
is the max over ranks; value = all ranks' neuron-steps / that time.

The default line also carries `c3` (config 3's network training step with
spike-input layers, the nn.Linear + lif_tuned step beside it and their spikes
compared bit for bit; data parallel under torchrun; --no-c3 skips it) and,
under torchrun, `tshard_parity` and `c4_tshard` (config 4 time-sharded over
the ranks, checked against single-GPU lif_tuned, with per-phase maxima and
the "maps" entry mode beside; --no-tshard skips them).

--impl reference times the reference's CPU path for the same workload: the
CPU oracle (oracle/, a C restatement of lifscan/fast.py's serial forward and
adjoint) on all host threads.  Under torchrun only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

T_STEPS = 1024
N_PER_GPU = 16384
BETA = 0.99
MU, SD = 0.05, 0.2
FWD_BYTES = 12   # read I, write U (or V) and S (fp32) per neuron-step
# lif_tuned's backward reads I, U[t-1], GS and writes Lam (GU is identically
# zero and S is recomputed bit-exactly from U and I); when its forward is the
# single pass it saves V (the pre-reset potential) instead of U and the
# backward reads V and GS only.
BWD_BYTES = 16
BWD_BYTES_V = 12
METRIC = "neuron-steps/s, lif_tuned fwd+bwd (B*N=16384/GPU, T=1024)"
UNIT = "neuron-steps/s"
FALLBACK_HBM_GBS = 6650.0
C4_T, C4_N, C4_MU, C4_SD = 1 << 20, 1024, 0.02, 0.1
C4_METRIC = "neuron-steps/s, fwd+bwd of one sequence (B*N=1024, T=2^20)"
C4_WORKLOAD = "c4: T=2^20, B*N=1024, beta=0.99, x~N(0.02,0.1^2), forward + backward"
L2_FLUSH_BYTES = 256 << 20
C1_T, C1_N, C1_BETA, C1_MU, C1_SD = 1024, 4096, 0.9, 0.1, 0.3
C1_METRIC = "neuron-steps/s, scan forward (B*N=4096/GPU, T=1024)"
C1_WORKLOAD = "c1: scan forward, B*N=4096 per GPU (B=16 x 256), T=1024, beta=0.9, x~N(0.1,0.3^2)"
C1_RING = 6  # input sets cycled by the c1 timing: 6 x 48 MiB > the 126 MB L2
C2_RING = 3  # input sets cycled by the c2 timing: each step touches 320 MiB


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", default="b200", choices=("b200", "reference"))
    p.add_argument("--mode", default="scan", choices=("scan", "serial", "auto"),
                   help="lif_tuned mode (default: the reference's default, scan)")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-c3", action="store_true",
                   help="default run: skip the config-3 network step sub-object")
    p.add_argument("--no-tshard", action="store_true",
                   help="under torchrun, skip the config-4 time-sharded parity check and timing of the default run")
    p.add_argument("--cpu-seconds", type=float, default=10.0)
    p.add_argument("--workload", default="c2", choices=("c1", "c2", "c3", "c4", "c5", "soft", "affine", "alif"),
                   help="c1: the scan forward of config 1 (B*N=4096, T=1024); "
                        "c2: lif_tuned fwd+bwd (the headline); c3: 700-256-256-20 network training step; "
                        "c4: T=2^20, B*N=1024 fwd+bwd, time-sharded over the GPUs; c5: sweep of B*N, T, beta; "
                        "soft: the soft-reset fitting layer (lif_soft) at config 2's shape and a long soft scan; "
                        "affine: the affine-reset layer (lif_affine) at config 2's shape and a long affine scan; "
                        "alif: the ALIF layer (alif) at config 2's shape and a long ALIF scan")
    p.add_argument("--c5-n", default="14,15,16,17,18,19,20,21,22",
                   help="c5: log2 of the total B*N values (split over the GPUs)")
    p.add_argument("--c5-t", default="256,1024,4096", help="c5: sequence lengths")
    return p.parse_args()


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def traffic_per_unit(kernel_key):
    """DRAM bytes per neuron-step of a kernel from a committed ncu summary
    (profiles/traffic.json), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
            d = json.load(f)
        return float(d[kernel_key]["dram_bytes_per_neuron_step"])
    except (OSError, KeyError, ValueError, TypeError):
        return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML during the timed
    region: once on entry, every `period` seconds from a thread, and once on
    exit, so that even a region of a few milliseconds has samples from its
    start and its end."""
    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}

    def __init__(self, index, period=0.005):
        self.index, self.period = index, period
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._lock = threading.Lock()
        self._t = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # NVML missing: no clock record
            self.ok = False

    def _sample(self):
        nv = self.nv
        try:
            mhz = nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)
            r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:  # a failed query leaves no sample
            return
        with self._lock:
            self.samples.append(mhz)
            for bit, name in self.REASONS.items():
                if r & bit:
                    self.reasons.add(name)

    def _run(self):
        while not self._stop.wait(self.period):
            self._sample()

    def __enter__(self):
        if self.ok:
            self._sample()
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join()
        if self.ok:
            self._sample()

    def record(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


class RingTimer:
    """Back-to-back timing of a step over a ring of input sets whose joint
    footprint exceeds L2, so every step reads inputs that are no longer in L2
    (the contract's "inputs larger than L2", instead of a flush per step).

    One CUDA graph holds one step per set (a full cycle of the ring), so the
    host launches one graph per cycle and the device runs the steps back to
    back; K steps are timed by one pair of CUDA events as floor(K / R)
    replays of the cycle graph plus K mod R replays of single-step graphs.
    `step_fns[r]()` runs one step on set r (warmed up before capture)."""

    def __init__(self, torch, dev, stream, lib, step_fns, barrier):
        self.torch, self.dev, self.stream, self.barrier = torch, dev, stream, barrier
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(2):
                for fn in step_fns:
                    fn()
        stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        self.single = []
        n0 = lib.lifb_kernel_launches()
        for fn in step_fns:
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                fn()
            self.single.append(gr)
        self.launches_per_step = (lib.lifb_kernel_launches() - n0) // len(step_fns)
        self.cycle = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.cycle):
            for fn in step_fns:
                fn()
        torch.cuda.synchronize(dev)
        self.R = len(step_fns)

    def run(self, steps):
        q, r = divmod(steps, self.R)
        for _ in range(q):
            self.cycle.replay()
        for i in range(r):
            self.single[i].replay()

    def ms_per_step(self, steps):
        torch = self.torch
        self.run(self.R)
        self.barrier()
        torch.cuda.synchronize(self.dev)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(self.stream)
        self.run(steps)
        b.record(self.stream)
        torch.cuda.synchronize(self.dev)
        self.barrier()
        return a.elapsed_time(b) / steps


def bind_numa(torch, dev):
    """Binds this process's CPUs to the NUMA node of its GPU (read from
    sysfs), so pinned host buffers allocated afterwards are first touched on
    that node.  Returns the node, or None when the platform does not say."""
    try:
        p = torch.cuda.get_device_properties(dev)
        bdf = f"{p.pci_domain_id:04x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        with open(f"/sys/bus/pci/devices/{bdf}/numa_node") as f:
            node = int(f.read().strip())
        if node < 0:
            return None
        with open(f"/sys/devices/system/node/node{node}/cpulist") as f:
            cpus = set()
            for part in f.read().strip().split(","):
                a, _, b = part.partition("-")
                cpus.update(range(int(a), int(b or a) + 1))
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
        return node
    except (OSError, ValueError, AttributeError):
        return None


def cpu_oracle_rate(T, N, seconds, want_bwd=True, mu=MU, sd=SD, beta=BETA):
    """Reference CPU path (C restatement of lifscan/fast.py serial forward +
    adjoint) on all host threads; repeats the full workload until `seconds`
    have elapsed (at least once).  Returns (neuron-steps/s, threads, sample)."""
    from oracle import oracle as O
    O.set_threads(os.cpu_count() or 1)  # all host threads (torchrun sets OMP_NUM_THREADS=1)
    I, u0, GS = O.gen_inputs(T, N, mu, sd, seed=0, grad=True)
    threads = O.num_threads()
    O.serial_forward(I[:64], beta, 1.0, 0.0, u0)  # warm the library
    done = 0
    t0 = time.perf_counter()
    while True:
        U, S = O.serial_forward(I, beta, 1.0, 0.0, u0)
        if want_bwd:
            O.serial_backward(I, u0, U, S, GS, None, beta, 1.0, 0.0, 4.0, True)
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    what = "serial forward + adjoint" if want_bwd else "serial forward"
    return done * T * N / el, threads, f"{done} x T={T}, N={N} ({what}) in {el:.1f} s"


SOFT_METRIC = "neuron-steps/s, soft-reset fitting layer lif_soft fwd+bwd (B*N=16384/GPU, T=1024)"
AFF_METRIC = "neuron-steps/s, affine-reset layer lif_affine fwd+bwd (B*N=16384/GPU, T=1024)"
ALIF_METRIC = "neuron-steps/s, ALIF layer alif fwd+bwd (B*N=16384/GPU, T=1024)"
C3_METRIC = "LIF neuron-steps/s, 700-256-256-20 training step (B=64/GPU, T=1024)"
C5_METRIC = "neuron-steps/s, lif_tuned fwd+bwd over the config-5 sweep (largest point)"


def _reference_network_step(O):
    """One training step of the config-3 network (700-256-256-20, B = 64,
    T = 1024, beta = 0.9, Kaiming-uniform Linear layers, leaky readout,
    cross-entropy, Adam) on the CPU: torch's CPU Linear layers around the
    oracle's serial LIF forward and adjoint (the C port of lifscan/fast.py).
    Returns (step function, LIF neuron-steps per step)."""
    import math

    import numpy as np
    import torch
    import torch.nn as nn

    from hard_resets_compose_b200.shdnet import synthetic_batch

    torch.set_num_threads(os.cpu_count() or 1)

    class OracleLIF(torch.autograd.Function):
        """Hard-reset LIF over [T, M] (spikes out); with theta = inf the
        leaky integrator (potential out, gradient on the potential)."""

        @staticmethod
        def forward(ctx, I, beta, theta):
            x = I.detach().contiguous().numpy()
            u0 = np.zeros(x.shape[1], np.float32)
            U, S = O.serial_forward(x, beta, theta, 0.0, u0)
            ctx.st = (x, u0, U, S, beta, theta)
            return torch.from_numpy(S if math.isfinite(theta) else U)

        @staticmethod
        def backward(ctx, g):
            x, u0, U, S, beta, theta = ctx.st
            gn = g.detach().contiguous().numpy()
            if math.isfinite(theta):
                lam = O.serial_backward(x, u0, U, S, gn, None, beta, theta, 0.0, 4.0, True)
            else:
                lam = O.serial_backward(x, u0, U, S, np.zeros_like(gn), gn, beta, theta, 0.0, 4.0, True)
            return torch.from_numpy(lam), None, None

    T, B, H, beta = 1024, 64, 256, 0.9
    torch.manual_seed(0)
    l1, l2, out = nn.Linear(700, H), nn.Linear(H, H), nn.Linear(H, 20)
    params = list(l1.parameters()) + list(l2.parameters()) + list(out.parameters())
    opt = torch.optim.Adam(params, lr=1e-3)
    x, y = synthetic_batch(T, B, seed=1000, device="cpu")

    def step():
        opt.zero_grad(set_to_none=True)
        s1 = OracleLIF.apply(l1(x).reshape(T, -1), beta, 1.0).reshape(T, B, H)
        s2 = OracleLIF.apply(l2(s1).reshape(T, -1), beta, 1.0).reshape(T, B, H)
        z = out(s2)
        yv = OracleLIF.apply(z.reshape(T, -1), beta, math.inf).reshape(T, B, 20).mean(0)
        nn.functional.cross_entropy(yv, y).backward()
        opt.step()

    return step, 2 * B * H * T


def run_reference(args, ws, rank):
    """The reference's CPU path for the chosen workload, on all host threads:
    the oracle (a C port of lifscan/fast.py and of the reset families' serial
    recurrences and adjoints) on a bounded sample of the workload, under the
    same metric as this workload's b200 line."""
    if rank != 0:
        return
    from oracle import oracle as O
    O.set_threads(os.cpu_count() or 1)  # all host threads (torchrun sets OMP_NUM_THREADS=1)
    wl = args.workload
    scaling = "weak"
    if wl == "c1":
        T, N = C1_T, C1_N
        I, u0 = O.gen_inputs(T, N, C1_MU, C1_SD, seed=0)

        def one_step():
            O.serial_forward(I, C1_BETA, 1.0, 0.0, u0)
        units = N * T
        metric, workload = C1_METRIC, C1_WORKLOAD
        sample = f"full workload per step (T={T}, N={N}), serial forward"
        path = "CPU oracle port of lifscan/fast.py serial_forward_nograd"
    elif wl == "c3":
        one_step, units = _reference_network_step(O)
        metric = C3_METRIC
        workload = "c3: 700-256-256-20 training step, B=64, T=1024, beta=0.9, leaky readout, Adam"
        sample = "the full training step (torch CPU Linear layers, oracle LIF forward and adjoint)"
        path = "torch CPU Linear layers + CPU oracle port of lifscan/fast.py's serial LIF and adjoint"
    else:
        if wl == "c4":
            # bounded sample of config 4: the first 2^17 of its 2^20 rows, all 1024 neurons
            T, N, mu, sd, beta = 1 << 17, C4_N, C4_MU, C4_SD, BETA
            metric, scaling, workload = C4_METRIC, "strong", C4_WORKLOAD
            sample = f"first {T} of {C4_T} rows per step (N={N}), serial forward + adjoint"
        elif wl == "c5":
            # bounded sample of the sweep's largest point (B*N = 2^22, T = 4096, beta = 0.99)
            T, N, mu, sd, beta = 4096, N_PER_GPU, 0.1, 0.3, 0.99
            metric = C5_METRIC
            workload = "c5: largest point B*N=2^22, T=4096, beta=0.99, x~N(0.1,0.3^2), fwd+bwd"
            sample = f"first {N} of {1 << 22} neurons per step (T={T}), serial forward + adjoint"
        else:
            T, N, mu, sd, beta = T_STEPS, N_PER_GPU, MU, SD, BETA
            metric = {"soft": SOFT_METRIC, "affine": AFF_METRIC, "alif": ALIF_METRIC}.get(wl, METRIC)
            workload = {"soft": "soft: lif_soft fwd+bwd with dbeta, beta=0.99, x~N(0.05,0.2^2)",
                        "affine": f"affine: lif_affine fwd+bwd with dbeta, dgamma, ddelta, beta=0.99, "
                                  f"gamma={AFF_GAMMA}, delta={AFF_DELTA}, x~N(0.05,0.2^2)",
                        "alif": f"alif: alif fwd+bwd with dbeta, drho, dq, dtheta0, beta=0.99, rho={ALIF_RHO}, "
                                f"q={ALIF_Q}, theta0=1, x~N(0.05,0.2^2)"}.get(
                wl, "c2: lif_tuned fwd+bwd, B*N=16384, T=1024, beta=0.99, x~N(0.05,0.2^2)")
            sample = f"full workload per step (T={T}, N={N}), serial forward + adjoint"
        I, u0, GS = O.gen_inputs(T, N, mu, sd, seed=0, grad=True)
        if wl in ("soft", "affine"):
            # the soft reset is the affine reset at gamma = 1, delta = -theta
            g, d = (1.0, -1.0) if wl == "soft" else (AFF_GAMMA, AFF_DELTA)
            path = "CPU oracle port of the affine-reset serial recurrence and adjoint with the parameter sums"

            def one_step():
                U, _ = O.aff_serial_forward(I, beta, 1.0, g, d, u0)
                O.aff_serial_backward(I, u0, U, GS, beta, 1.0, g, 4.0)
        elif wl == "alif":
            path = "CPU oracle port of the ALIF serial recurrence and adjoint with the parameter sums"

            def one_step():
                U, W, S = O.alif_serial_forward(I, beta, ALIF_RHO, ALIF_Q, 1.0, 0.0, u0, u0)
                O.alif_serial_backward(I, u0, u0, U, W, S, GS, beta, ALIF_RHO, ALIF_Q, 1.0, 4.0)
        else:
            path = "CPU oracle port of lifscan/fast.py serial_forward_nograd + serial_backward"

            def one_step():
                U, S = O.serial_forward(I, beta, 1.0, 0.0, u0)
                O.serial_backward(I, u0, U, S, GS, None, beta, 1.0, 0.0, 4.0, True)
        units = N * T
    for _ in range(max(args.warmup, 0)):
        one_step()
    ts = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        one_step()
        ts.append(time.perf_counter() - t0)
    ms = 1e3 * sum(ts) / len(ts)
    value = units / (ms / 1e3)
    cores = O.num_threads()
    line = {
        "impl": "reference", "metric": metric, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": workload, "path": path},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_c1(args, ws, rank, local):
    """Config 1: the scan forward (spikes and membrane potentials) of
    B*N = 4096 neurons per GPU over T = 1024 rows, x ~ N(0.1, 0.3^2),
    beta = 0.9, u0 = 0.  The step is scan_forward_auto, the library's path
    for this shape; the map scan (scan_forward_v3 with the reference's C = 64,
    K = 16, the block-level kernel), the lead-in block scan and the single
    serial pass are timed beside it.  Batch-sharded under torchrun (weak
    scaling, no collective).  Every path is checked bit for bit against the
    serial pass on the device before timing.

    A step's working set (48 MiB) fits in L2, so the timed region runs K
    steps back to back over a ring of C1_RING input sets (their inputs and
    outputs together exceed L2: each step's input was last touched
    C1_RING - 1 steps earlier, with more than L2's capacity of other traffic
    since), one pair of CUDA events around all K.  Each path is also timed as
    an isolated call after an L2 flush (the event pair then also holds the
    launch's fixed latency, about 6 us measured for an empty kernel)."""
    import datetime

    import torch
    import torch.distributed as dist

    from hard_resets_compose_b200 import _lib
    from hard_resets_compose_b200 import lifscan as L

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    lib = _lib.load()
    T, N, beta = C1_T, C1_N, C1_BETA
    g = torch.Generator().manual_seed(100 + rank)
    I_hs = [(C1_MU + C1_SD * torch.randn(T, N, generator=g)).float() for _ in range(C1_RING)]
    u0_h = torch.zeros(N)
    Is = [x.to(dev) for x in I_hs]
    u0 = u0_h.to(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    evict = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if ws > 1:
            dist.barrier()

    def max_over_ranks(x):
        if ws == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    Lb, Wb = L.block_leadin(T, N, beta)

    def path_fns(I):
        f = {"auto": lambda: L.scan_forward_auto(I, beta, 1.0, 0.0, u0),
             "map_scan_v3_C64_K16": lambda: L.scan_forward_v3(I, beta, 1.0, 0.0, u0, C=64, K=16),
             "serial": lambda: L.serial_forward(I, beta, 1.0, 0.0, u0)}
        if Lb:
            f[f"leadin_block_L{Lb}_W{Wb}"] = lambda: L.scan_forward_spec(I, beta, 1.0, 0.0, u0, L=Lb, W=Wb)
        return f
    ring = [path_fns(I) for I in Is]
    parity = True
    for fns in ring[:2]:
        Us, Ss = fns["serial"]()
        for name, fn in fns.items():
            U_, S_ = fn()
            parity &= bool(torch.equal(U_.view(torch.int32), Us.view(torch.int32)) and
                           torch.equal(S_.view(torch.int32), Ss.view(torch.int32)))
    del U_, S_, Us, Ss

    def isolated_ms(replay, steps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        barrier()
        torch.cuda.synchronize(dev)
        for a, b in evs:
            flush.fill_(1.0)
            torch.sum(evict, dim=0, out=sink)
            a.record(stream)
            replay()
            b.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        return sum(a.elapsed_time(b) for a, b in evs) / steps

    for _ in range(max(args.warmup, 3)):
        for fns in ring:
            for fn in fns.values():
                fn()
    torch.cuda.synchronize(dev)
    per_path = {}
    clk_rec = None
    launches = 0
    for k in ring[0]:
        rt = RingTimer(torch, dev, stream, lib, [fns[k] for fns in ring], barrier)
        nl = rt.launches_per_step
        if k == "auto":
            with ClockSampler(local) as clk:
                ms = rt.ms_per_step(args.steps)
            clk_rec = clk.record()
            launches = nl * args.steps
        else:
            ms = rt.ms_per_step(args.steps)
        ms = max_over_ranks(ms)
        ms_iso = max_over_ranks(isolated_ms(rt.single[0].replay, max(args.steps // 2, 5)))
        per_path[k] = {"ms": ms, "value": N * T * ws / (ms / 1e3), "launches_per_call": nl,
                       "gbs": FWD_BYTES * N * T / (ms / 1e3) / 1e9, "isolated_call_ms": ms_iso}
        del rt
    ms = per_path["auto"]["ms"]
    units = N * T * ws
    value = units / (ms / 1e3)
    hbm, peak_kind = peaks()
    for v in per_path.values():
        v["frac"] = v["gbs"] / hbm
    tpu = traffic_per_unit("c1_auto")
    roofline = {"bound": "hbm", "kernel": "scan_forward_auto at config 1 (its launches per call: "
                f"{per_path['auto']['launches_per_call']})", "achieved": per_path["auto"]["gbs"], "peak": hbm,
                "peak_source": peak_kind, "unit": "GB/s", "frac": per_path["auto"]["frac"],
                "traffic": (tpu * N * T) if tpu is not None else None, "algorithmic_bytes": FWD_BYTES * N * T}

    e2e = None
    if not args.no_e2e:
        I_pin = I_hs[0].pin_memory()
        U_pin = torch.empty(T, N).pin_memory()
        S_pin = torch.empty(T, N).pin_memory()

        def e2e_step():
            Id = I_pin.to(dev, non_blocking=True)
            U_, S_ = L.scan_forward_auto(Id, beta, 1.0, 0.0, u0)
            U_pin.copy_(U_, non_blocking=True)
            S_pin.copy_(S_, non_blocking=True)
        for _ in range(3):
            e2e_step()
        n_e = max(args.steps // 2, 5)
        barrier()
        torch.cuda.synchronize(dev)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(n_e):
            e2e_step()
        b.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        ms_e = max_over_ranks(a.elapsed_time(b) / n_e)
        e2e = {"value": units / (ms_e / 1e3), "unit": UNIT, "ms_per_step": ms_e,
               "h2d_bytes_per_step": T * N * 4, "d2h_bytes_per_step": 2 * T * N * 4,
               "api": "pinned host I -> .to(cuda) -> scan_forward_auto -> U, S copied to pinned host buffers, "
                      "steps back to back"}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        v, threads, sample = cpu_oracle_rate(T, N, args.cpu_seconds, want_bwd=False, mu=C1_MU, sd=C1_SD, beta=beta)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}
    if rank == 0:
        print(json.dumps({
            "metric": C1_METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded torch.Generator, config 1 shape)",
            "config": {"workload": C1_WORKLOAD, "global_neurons": N * ws, "seq_len": T,
                       "parallelism": f"batch-sharded x{ws}, no collective",
                       "step": "scan_forward_auto; one CUDA graph holds one step per input set of the ring",
                       "l2": f"inputs larger than L2: {args.steps} steps back to back over a ring of {C1_RING} input "
                             f"sets ({C1_RING} x 48 MiB of I, U, S), one event pair around all of them; "
                             "isolated_call_ms: one call after an L2 flush, its own event pair (launch latency "
                             "included)"},
            "parity_bit_exact_vs_serial": parity, "paths": per_path,
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "clocks": clk_rec}), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_sweep(args, ws, rank, local):
    """Config 5: forward and forward+backward over B*N in 2^14..2^22 (total,
    batch-sharded over the GPUs), T in {256, 1024, 4096}, beta in {0.9, 0.99},
    x ~ N(0.1, 0.3^2).  Each point times the library calls lif_tuned makes
    (scan_forward_auto; scan_backward_auto with S recomputed and no GU) with
    CUDA events, L2 flushed before every timed call; points whose tensors do
    not fit this GPU (5 [T, N] fp32 tensors for fwd+bwd) are reported as
    skipped.  One JSON line: every point, and the headline = the largest
    point's fwd+bwd throughput."""
    import datetime

    import torch
    import torch.distributed as dist

    from hard_resets_compose_b200 import _lib
    from hard_resets_compose_b200 import lifscan as L

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    _lib.load()
    hbm, peak_kind = peaks()
    free_bytes = torch.cuda.mem_get_info(dev)[1]
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    evict = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)

    def flush_l2():
        flush.fill_(1.0)
        torch.sum(evict, dim=0, out=sink)

    def max_over_ranks(v):
        if ws == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def timed(fn, reps):
        fn()
        ms = []
        for _ in range(reps):
            flush_l2()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            b.record(stream)
            b.synchronize()
            ms.append(a.elapsed_time(b))
        return statistics.median(ms)

    points = []
    reps = max(args.steps, 3)
    with ClockSampler(local) as clk:
        for lg in (int(v) for v in args.c5_n.split(",")):
            for T in (int(v) for v in args.c5_t.split(",")):
                for beta in (0.9, 0.99):
                    n_tot = 1 << lg
                    N = n_tot // ws
                    need = 5 * T * N * 4 + (1 << 30)
                    pt = {"N": n_tot, "T": T, "beta": beta}
                    fits = float(need <= 0.9 * free_bytes)
                    if ws > 1:
                        t = torch.tensor([fits], device=dev)
                        dist.all_reduce(t, op=dist.ReduceOp.MIN)
                        fits = float(t.item())
                    if not fits:
                        pt["skipped"] = f"needs {need / 2**30:.0f} GiB per GPU for fwd+bwd"
                        points.append(pt)
                        continue
                    g = torch.Generator(device=dev).manual_seed(5000 + lg * 7 + T + rank)
                    I = torch.empty(T, N, device=dev).normal_(0.1, 0.3, generator=g)
                    GS = torch.empty(T, N, device=dev).normal_(0.0, 1.0, generator=g)
                    u0 = torch.zeros(N, device=dev)
                    out = {}

                    vpath = L._single_pass(T, N, "scan")  # what lif_tuned(mode="scan") runs here

                    def fwd():
                        out.clear()
                        out["fwd"] = L.serial_forward_v(I, beta, 1.0, 0.0, u0) if vpath else \
                            L.scan_forward_auto(I, beta, 1.0, 0.0, u0)

                    def fwd_bwd():  # at most I, GS, U (or V), S and Lam live
                        out.clear()
                        if vpath:
                            V_, _ = L.serial_forward_v(I, beta, 1.0, 0.0, u0)
                            out["lam"] = L.lif_backward_v(V_, GS, beta, 1.0, 4.0, C=L.scan_chunk_bwd(T, N))
                        else:
                            U_, _ = L.scan_forward_auto(I, beta, 1.0, 0.0, u0)
                            out["lam"] = L.scan_backward_auto(I, u0, U_, None, GS, None, beta, 1.0, 0.0, 4.0)

                    ms_f = max_over_ranks(timed(fwd, reps))
                    ms_fb = max_over_ranks(timed(fwd_bwd, reps))
                    units = T * n_tot
                    step_bytes = FWD_BYTES + (BWD_BYTES_V if vpath else BWD_BYTES)
                    gbs_f = FWD_BYTES * T * N / (ms_f / 1e3) / 1e9
                    gbs_fb = step_bytes * T * N / (ms_fb / 1e3) / 1e9
                    pt.update(fwd_ms=ms_f, fwd_value=units / (ms_f / 1e3), fwd_frac=gbs_f / hbm,
                              fwd_bwd_ms=ms_fb, fwd_bwd_value=units / (ms_fb / 1e3), fwd_bwd_frac=gbs_fb / hbm,
                              forward_segments=list(L.spec_segment(T, N)), bwd_chunk=L.scan_chunk_bwd(T, N),
                              saved="V" if vpath else "U", fwd_bwd_bytes_per_neuron_step=step_bytes)
                    points.append(pt)
                    del I, GS, u0, out
                    torch.cuda.empty_cache()
    done = [p for p in points if "skipped" not in p]
    head = max(done, key=lambda p: (p["N"] * p["T"], p["beta"])) if done else None
    if rank == 0:
        print(json.dumps({
            "metric": C5_METRIC,
            "value": head["fwd_bwd_value"] if head else None, "unit": UNIT, "n_gpus": ws, "steps": reps,
            "warmup": 1, "ms_per_step": head["fwd_bwd_ms"] if head else None, "higher_is_better": True,
            "scaling": "weak" if ws > 1 else "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded CUDA torch.Generator, x ~ N(0.1, 0.3^2), upstream gradient N(0, 1))",
            "config": {"workload": "c5: sweep B*N x T x beta, fwd and fwd+bwd", "parallelism":
                       f"batch-sharded x{ws}, no collective" if ws > 1 else "one GPU",
                       "l2": "flushed before every timed call (256 MiB written, 256 MiB read)",
                       "peak": hbm, "peak_source": peak_kind},
            "points": points, "clocks": clk.record()}), flush=True)
    if ws > 1:
        dist.destroy_process_group()


# affine workload: the reset u <- gamma*v + delta at one of the reference's
# test points (lifscan tests/test_affine.py:7)
AFF_GAMMA, AFF_DELTA = 0.3, -0.1
# alif workload: the "lsnn" neuron class of lifscan tests/test_alif.py:10
ALIF_RHO, ALIF_Q = 0.995, 0.9


def run_reset_family(args, ws, rank, local, family):
    """The soft-reset model (family "soft": subtractive reset; lifscan/fit.py:
    93-121 lif_soft, lifscan/triton_soft.py soft_scan_forward), the
    affine-reset model (family "affine": u <- gamma*v + delta, gamma = 0.3,
    delta = -0.1; lifscan/triton_affine.py lif_affine, aff_scan_forward) or the
    ALIF model (family "alif": rho = 0.995, q = 0.9; lifscan/triton_alif.py
    alif, alif_scan_forward): the layer's forward + backward (spikes out;
    gradients for I, u0 and beta, and for gamma and delta, or for w0, rho, q
    and theta0) at config 2's shape (B*N = 16384 per GPU,
    T = 1024, x ~ N(0.05, 0.2^2), beta = 0.99), issued eagerly; and the exact
    scan forward at T = 2^18, N = 1024 (x ~ N(0.02, 0.1^2)) beside the serial
    pass it replaces (for ALIF also the two-level adjoint with the parameter
    sums at that length, beside the one reverse sweep)."""
    if rank != 0:
        return  # one-GPU workload: under torchrun only rank 0 measures (its line says n_gpus = 1)
    import torch

    from hard_resets_compose_b200 import _lib
    from hard_resets_compose_b200 import affine as A
    from hard_resets_compose_b200 import alif as AL
    from hard_resets_compose_b200 import fit
    from hard_resets_compose_b200 import lifscan as L
    from hard_resets_compose_b200 import soft as TS

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    lib = _lib.load()
    T, N = T_STEPS, N_PER_GPU
    g = torch.Generator(device=dev).manual_seed(7000 + rank)
    I = torch.empty(T, N, device=dev).normal_(MU, SD, generator=g)
    GS = torch.empty(T, N, device=dev).normal_(0.0, 1.0, generator=g)
    u0 = torch.zeros(N, device=dev)
    Iq = I.clone().requires_grad_(True)
    b = torch.tensor(BETA, device=dev, requires_grad=True)
    gm = torch.tensor(AFF_GAMMA, device=dev, requires_grad=True)
    dl = torch.tensor(AFF_DELTA, device=dev, requires_grad=True)
    rh = torch.tensor(ALIF_RHO, device=dev, requires_grad=True)
    qq = torch.tensor(ALIF_Q, device=dev, requires_grad=True)
    th = torch.tensor(1.0, device=dev, requires_grad=True)
    w0 = torch.zeros(N, device=dev)
    stream = torch.cuda.current_stream(dev)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)
    evict = torch.ones(L2_FLUSH_BYTES // 4, device=dev)
    sink = torch.empty((), device=dev)
    soft = family == "soft"

    def step():
        Iq.grad = None
        b.grad = gm.grad = dl.grad = rh.grad = qq.grad = th.grad = None
        if soft:
            S = fit.lif_soft(Iq, u0, b, 1.0, 4.0)
        elif family == "alif":
            S, _, _ = AL.alif(Iq, u0, w0, b, rh, qq, th, fwd="serial", bwd="serial")
        else:
            S = A.lif_affine(Iq, u0, b, gm, dl, theta=1.0, alpha=4.0, mode="serial")
        torch.autograd.backward(S, GS)

    def timed(fn, steps):
        ms = []
        for _ in range(steps):
            flush.fill_(1.0)
            torch.sum(evict, dim=0, out=sink)
            a = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            e.record(stream)
            e.synchronize()
            ms.append(a.elapsed_time(e))
        return statistics.median(ms)

    def timed_queued(fn, steps):
        """Device time of one call of fn: every iteration (L2 flush, event,
        call, event) is queued before the host waits, so the host prepares
        each call while the GPU runs the flush before it, and the events time
        the call's own kernels (fn must not synchronise)."""
        ev = []
        for _ in range(steps):
            flush.fill_(1.0)
            torch.sum(evict, dim=0, out=sink)
            a = torch.cuda.Event(enable_timing=True)
            e = torch.cuda.Event(enable_timing=True)
            a.record(stream)
            fn()
            e.record(stream)
            ev.append((a, e))
        torch.cuda.synchronize(dev)
        return statistics.median(a.elapsed_time(e) for a, e in ev)

    # eager: the layer reads beta (a CUDA tensor) on the host, like the
    # reference's (lifscan/fit.py:98, triton_affine.py:219), which rules out
    # graph capture
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    n0 = lib.lifb_kernel_launches()
    with ClockSampler(local) as clk:
        ms = timed(step, args.steps)
    launches = (lib.lifb_kernel_launches() - n0) // max(args.steps, 1)
    if soft:
        # the layer's single-pass path: the soft reset as the affine reset
        # (gamma = 1, delta = -theta), V saved, dbeta summed in the adjoint sweep
        fwd = lambda: A.aff_serial_forward_v(I, BETA, 1.0, 1.0, -1.0, u0)  # noqa: E731
        V, S = fwd()
        bwd = lambda: A.aff_adjoint_v(V, u0, GS, BETA, 1.0, 1.0, -1.0, 4.0)  # noqa: E731
        serial_long = lambda x, z: L.soft_serial_forward(x, BETA, 1.0, z)  # noqa: E731
        scan_long = lambda x, z: TS.soft_scan_forward(x, BETA, 1.0, z)  # noqa: E731
    elif family == "alif":
        fwd = lambda: AL.alif_serial_forward(I, BETA, ALIF_RHO, ALIF_Q, 1.0, 0.0, u0, w0)  # noqa: E731
        U, W, S = fwd()
        bwd = lambda: AL._alif_bwd(I, u0, w0, U, W, None, GS, BETA, ALIF_RHO, ALIF_Q, 1.0, 4.0,  # noqa: E731
                                   False, True)
        serial_long = lambda x, z: AL.alif_serial_forward(x, BETA, ALIF_RHO, ALIF_Q, 1.0, 0.0, z, z)  # noqa: E731
        scan_long = lambda x, z: AL.alif_scan_forward(x, BETA, ALIF_RHO, ALIF_Q, 1.0, 0.0, z, z, None,  # noqa: E731
                                                      0.1, C=128)
    else:
        # the layer's single-pass path: forward writes V and S, the adjoint
        # reads V and gS and sums the parameter gradients in the same sweep
        fwd = lambda: A.aff_serial_forward_v(I, BETA, 1.0, AFF_GAMMA, AFF_DELTA, u0)  # noqa: E731
        V, S = fwd()
        bwd = lambda: A.aff_adjoint_v(V, u0, GS, BETA, 1.0, AFF_GAMMA, AFF_DELTA, 4.0)  # noqa: E731
        serial_long = lambda x, z: A.aff_serial_forward(x, BETA, 1.0, AFF_GAMMA, AFF_DELTA, z)  # noqa: E731
        scan_long = lambda x, z: A.aff_scan_forward(x, BETA, 1.0, AFF_GAMMA, AFF_DELTA, z)  # noqa: E731
    ms_f = timed_queued(fwd, args.steps)
    ms_b = timed_queued(bwd, args.steps)
    hbm, peak_kind = peaks()
    # soft and affine layers: forward 12 B (I in; V, S out), adjoint with the
    # parameter sums 12 B (V, GS in; Lam out).  ALIF layer: forward 16 B (I in;
    # U, W, S out), adjoint with the parameter sums 20 B (I, U[t-1], W[t-1],
    # GS in; LV out)
    fwd_bytes, bwd_bytes = {"soft": (12, 12), "affine": (12, 12), "alif": (16, 20)}[family]
    layer_bytes = fwd_bytes + bwd_bytes
    Tl, Nl = 1 << 18, 1024
    gl = torch.Generator(device=dev).manual_seed(7100 + rank)
    Il = torch.empty(Tl, Nl, device=dev).normal_(0.02, 0.1, generator=gl)
    u0l = torch.zeros(Nl, device=dev)
    ms_serial_long = timed(lambda: serial_long(Il, u0l), 3)
    ms_scan_long = timed(lambda: scan_long(Il, u0l), 3)
    long_adj = None
    if family == "alif":
        # the two-level adjoint with the parameter sums over the long sequence
        # (chunk maps composed, carried and replayed), beside the one sweep
        Ul, Wl, _ = AL.alif_serial_forward(Il, BETA, ALIF_RHO, ALIF_Q, 1.0, 0.0, u0l, u0l)
        GSl = torch.empty(Tl, Nl, device=dev).normal_(0.0, 1.0, generator=gl)

        def adj(chunked):
            return lambda: AL._alif_bwd(Il, u0l, u0l, Ul, Wl, None, GSl, BETA, ALIF_RHO, ALIF_Q, 1.0, 4.0,
                                        False, True, chunked=chunked)
        ms_adj_scan = timed_queued(adj(True), 3)
        ms_adj_sweep = timed_queued(adj(False), 3)
        long_adj = {"T": Tl, "N": Nl, "two_level_ms": ms_adj_scan, "one_sweep_ms": ms_adj_sweep,
                    "two_level_value": Tl * Nl / (ms_adj_scan / 1e3)}
        del Ul, Wl, GSl
    units = T * N
    if soft:
        metric = SOFT_METRIC
        workload = "soft: lif_soft (gradients for I, u0, beta), beta=0.99, x~N(0.05,0.2^2)"
    elif family == "alif":
        metric = ALIF_METRIC
        workload = (f"alif: alif fwd=serial (gradients for I, u0, w0, beta, rho, q, theta0), beta=0.99, "
                    f"rho={ALIF_RHO}, q={ALIF_Q}, theta0=1, x~N(0.05,0.2^2)")
    else:
        metric = AFF_METRIC
        workload = (f"affine: lif_affine mode=serial (gradients for I, u0, beta, gamma, delta), beta=0.99, "
                    f"gamma={AFF_GAMMA}, delta={AFF_DELTA}, x~N(0.05,0.2^2)")
    if rank == 0:
        print(json.dumps({
            "metric": metric,
            "value": units / (ms / 1e3), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded CUDA torch.Generator, config 2 shape)",
            "config": {"workload": workload, "gpus": f"one GPU (rank 0 of {ws})" if ws > 1 else "one GPU",
                       "step": "forward + torch.autograd.backward, issued eagerly (host overhead included)",
                       "l2": "flushed before every timed call (256 MiB written, 256 MiB read)"},
            "fwd": {"ms": ms_f, "bytes_per_unit": fwd_bytes, "gbs": fwd_bytes * units / (ms_f / 1e3) / 1e9,
                    "frac": fwd_bytes * units / (ms_f / 1e3) / 1e9 / hbm},
            "bwd": {"ms": ms_b, "bytes_per_unit": bwd_bytes, "gbs": bwd_bytes * units / (ms_b / 1e3) / 1e9,
                    "frac": bwd_bytes * units / (ms_b / 1e3) / 1e9 / hbm},
            "kernels_ms": ms_f + ms_b,
            "roofline": {"bound": "hbm", "kernel": "whole layer step (forward, adjoint, parameter reduction)",
                         "achieved": layer_bytes * units / (ms / 1e3) / 1e9, "peak": hbm, "peak_source": peak_kind,
                         "unit": "GB/s", "frac": layer_bytes * units / (ms / 1e3) / 1e9 / hbm, "traffic": None},
            "long_scan": {"T": Tl, "N": Nl, "serial_ms": ms_serial_long, "scan_ms": ms_scan_long,
                          "scan_value": Tl * Nl / (ms_scan_long / 1e3)},
            **({"long_adjoint": long_adj} if long_adj else {}),
            "gpu_launches": launches * args.steps, "clocks": clk.record()}), flush=True)


def run_long(args, ws, rank, local):
    """Config 4: one sequence of T = 2^20 rows, B*N = 1024 neurons,
    x ~ N(0.02, 0.1^2), beta = 0.99, forward + backward (spikes out, upstream
    gradient N(0, 1) on the spikes).  One GPU: lif_tuned (mode "scan", the
    library's long-sequence policy).  N GPUs: lif_tshard, rank r owning rows
    [r*T/N, (r+1)*T/N) (strong scaling: the total work is fixed), with the
    all-gathers of the time-sharded protocol over NCCL."""
    import datetime

    import torch
    import torch.distributed as dist

    from hard_resets_compose_b200 import _lib
    from hard_resets_compose_b200 import lifscan as L
    from hard_resets_compose_b200 import tshard

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    lib = _lib.load()
    N, T = C4_N, C4_T // ws
    g = torch.Generator(device=dev).manual_seed(4000 + rank)
    I = (C4_MU + C4_SD * torch.randn(T, N, generator=g, device=dev)).float()
    GS = torch.randn(T, N, generator=g, device=dev).float()
    u0 = torch.zeros(N, device=dev)
    Iq = I.clone().requires_grad_(True)
    stream = torch.cuda.current_stream(dev)
    comm = tshard.TorchComm() if ws > 1 else None
    ops = tshard.CudaSliceOps(T, N, dev, BETA, 1.0, 0.0) if ws > 1 else None

    def lif(x, u):
        if ws > 1:
            return tshard.lif_tshard(x, u, beta=BETA, ops=ops, comm=comm)
        return L.lif_tuned(x, u, beta=BETA, mode="scan")

    def step(x=Iq, G=GS, mid=None):
        x.grad = None
        S = lif(x, u0)
        if mid is not None:
            mid.record(stream)
        torch.autograd.backward(S, G)
        return S

    def max_over_ranks(v):
        if ws == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def barrier():
        if ws > 1:
            dist.barrier()

    for _ in range(max(args.warmup, 3)):
        step()
    steps = args.steps
    evs = [tuple(torch.cuda.Event(enable_timing=True) for _ in range(3)) for _ in range(steps)]
    barrier()
    torch.cuda.synchronize(dev)
    n0 = lib.lifb_kernel_launches()
    with ClockSampler(local) as clk:
        for a, m, b in evs:
            a.record(stream)
            step(mid=m)
            b.record(stream)
        torch.cuda.synchronize(dev)
    launches = lib.lifb_kernel_launches() - n0
    barrier()
    ms = max_over_ranks(sum(a.elapsed_time(b) for a, _, b in evs) / steps)
    ms_f = max_over_ranks(sum(a.elapsed_time(m) for a, m, _ in evs) / steps)
    ms_b = max_over_ranks(sum(m.elapsed_time(b) for _, m, b in evs) / steps)
    units = C4_T * N
    value = units / (ms / 1e3)
    hbm, peak_kind = peaks()
    phases = None
    if ws > 1:
        # one more step through the protocol functions with CUDA-event marks at
        # the end of each phase (untimed above); per phase the max over ranks
        for _ in range(2):  # the first direct call warms its allocations; the second is recorded
            tl = []
            U_, _, entry_ = tshard.tshard_forward(I, u0, ops, comm, timeline=tl)
            tshard.tshard_backward(I, entry_, U_, GS, ops, comm, BETA, timeline=tl)
            torch.cuda.synchronize(dev)
            del U_, entry_
        mine = [(tl[i][0], tl[i - 1][1].elapsed_time(tl[i][1])) for i in range(1, len(tl))]
        every = [None] * ws
        dist.all_gather_object(every, mine)
        per_phase = {}
        for lst in every:
            for name, v in lst:
                per_phase[name] = round(max(per_phase.get(name, 0.0), v), 4)
        phases = {"note": "one extra step through tshard_forward/backward (after one warm-up), CUDA events at the end of each "
                          "phase; per phase the max over ranks (rank 0 has no repair phase)",
                  "ms": per_phase, "step_ms_max": round(max(sum(v for _, v in lst) for lst in every), 4)}
    # algorithmic bytes of this rank's rows: forward 12 B, backward 16 B per neuron-step
    fwd_gbs = FWD_BYTES * T * N / (ms_f / 1e3) / 1e9
    bwd_gbs = BWD_BYTES * T * N / (ms_b / 1e3) / 1e9
    dom = ("fwd", ms_f, fwd_gbs, FWD_BYTES) if ms_f >= ms_b else ("bwd", ms_b, bwd_gbs, BWD_BYTES)
    roofline = {"bound": "hbm", "kernel": f"{dom[0]} phase of the step (all its launches)", "achieved": dom[2],
                "peak": hbm, "peak_source": peak_kind, "unit": "GB/s", "frac": dom[2] / hbm, "traffic": None,
                "algorithmic_bytes": dom[3] * T * N,
                "step_frac": (FWD_BYTES + BWD_BYTES) * T * N / (ms / 1e3) / 1e9 / hbm}

    e2e = None
    if not args.no_e2e:
        I_p = I.cpu().pin_memory()
        G_p = GS.cpu().pin_memory()
        S_p = torch.empty(T, N).pin_memory()
        dI_p = torch.empty(T, N).pin_memory()

        def e2e_step():
            Id = I_p.to(dev, non_blocking=True).requires_grad_(True)
            Gd = G_p.to(dev, non_blocking=True)
            S_ = step(Id, Gd)
            S_p.copy_(S_.detach(), non_blocking=True)
            dI_p.copy_(Id.grad, non_blocking=True)
        e2e_step()
        n_e = max(min(steps, 3), 1)
        ee = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n_e)]
        barrier()
        torch.cuda.synchronize(dev)
        for a, b in ee:
            a.record(stream)
            e2e_step()
            b.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        ms_e = max_over_ranks(sum(a.elapsed_time(b) for a, b in ee) / n_e)
        e2e = {"value": units / (ms_e / 1e3), "unit": UNIT, "ms_per_step": ms_e,
               "h2d_bytes_per_step": 2 * T * N * 4 * ws, "d2h_bytes_per_step": 2 * T * N * 4 * ws,
               "api": "pinned host slices -> .to(cuda) -> lif_tshard / lif_tuned + autograd.backward -> S, dI "
                      "copied back (all ranks)"}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        v, threads, sample = cpu_oracle_rate(1 << 17, N, args.cpu_seconds, mu=C4_MU, sd=C4_SD)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": sample + f" (the first 2^17 of the {C4_T} rows)"}
    if rank == 0:
        print(json.dumps({
            "metric": C4_METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded CUDA torch.Generator, config 4 shape)",
            "config": {"workload": C4_WORKLOAD, "seq_len": C4_T, "neurons": N,
                       "parallelism": f"time-sharded x{ws} (NCCL all-gathers)" if ws > 1 else "one GPU",
                       "path": "lif_tshard (entry_mode='speculate')" if ws > 1 else "lif_tuned(mode='scan')",
                       "forward_segments": list(L.spec_segment(T, N)),
                       "l2": "inputs (4 GiB per tensor / N) larger than L2"},
            "fwd": {"ms": ms_f, "gbs": fwd_gbs, "frac": fwd_gbs / hbm},
            "bwd": {"ms": ms_b, "gbs": bwd_gbs, "frac": bwd_gbs / hbm},
            "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "phases": phases, "clocks": clk.record()}), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


def c4_time_sharded(args, ws, rank, dev, lib):
    """Under torchrun (ws > 1) the default run also runs config 4's
    time-sharded scan (lif_tshard: rank r owns rows [r*T/ws, (r+1)*T/ws) of
    the 2^20-row sequence) and checks it against the whole sequence through
    single-GPU lif_tuned on every rank: U and S of the rank's rows bit for bit,
    dI within 1e-5 relative over all ranks, du0 within 1e-5.  Returns
    (tshard_parity, c4_tshard) for the JSON line: the parity verdict (every
    rank agreeing) and the timings (step max over ranks, per-phase maxima, the
    1-GPU step and the strong-scaling efficiency against it)."""
    import torch
    import torch.distributed as dist

    from hard_resets_compose_b200 import lifscan as L
    from hard_resets_compose_b200 import tshard

    stream = torch.cuda.current_stream(dev)
    N, T = C4_N, C4_T
    Ts = T // ws
    r0, r1 = rank * Ts, (rank + 1) * Ts
    g = torch.Generator(device=dev).manual_seed(4000)  # the same sequence on every rank
    I = (C4_MU + C4_SD * torch.randn(T, N, generator=g, device=dev)).float()
    GS = torch.randn(T, N, generator=g, device=dev).float()
    u0 = torch.zeros(N, device=dev)

    def all_max(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def all_sum(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def event_ms(fn, steps):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        dist.barrier()
        torch.cuda.synchronize(dev)
        for a, b in evs:
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize(dev)
        dist.barrier()
        return sum(a.elapsed_time(b) for a, b in evs) / steps

    # the whole sequence on this GPU: lif_tuned's forward potentials and gradients
    U1, S1 = L.scan_forward_auto(I, BETA, 1.0, 0.0, u0)
    Iq = I.clone().requires_grad_(True)
    u0q = u0.clone().requires_grad_(True)

    def step1():
        Iq.grad = None
        u0q.grad = None
        S_ = L.lif_tuned(Iq, u0q, beta=BETA, mode="scan")
        torch.autograd.backward(S_, GS)
        return S_
    S_layer = step1()
    s_layer_ok = bool(torch.equal(S_layer.detach().view(torch.int32), S1.view(torch.int32)))
    del S_layer
    dI1 = Iq.grad[r0:r1].clone()
    du01 = u0q.grad.clone()
    for _ in range(2):
        step1()
    ms1 = all_max(event_ms(step1, 3))
    del Iq, u0q

    Is = I[r0:r1].contiguous()
    GSs = GS[r0:r1].contiguous()
    U1s = U1[r0:r1].contiguous()
    S1s = S1[r0:r1].contiguous()
    del I, GS, U1, S1
    ops = tshard.CudaSliceOps(Ts, N, dev, BETA, 1.0, 0.0)
    comm = tshard.TorchComm()
    info = {}
    Us, Ss, entry = tshard.tshard_forward(Is, u0, ops, comm, info=info)
    Lam, du0 = tshard.tshard_backward(Is, entry, Us, GSs, ops, comm, BETA)
    ok = s_layer_ok and bool(torch.equal(Us.view(torch.int32), U1s.view(torch.int32)) and
                             torch.equal(Ss.view(torch.int32), S1s.view(torch.int32)))
    num = all_sum(float(((Lam.double() - dI1.double()) ** 2).sum()))
    den = all_sum(float((dI1.double() ** 2).sum()))
    dI_rel = (num / den) ** 0.5 if den > 0 else 0.0
    du0_rel = float((du0 - du01).norm() / du01.norm()) if rank == 0 else 0.0
    du0_rel = all_max(du0_rel)
    ok = ok and dI_rel <= 1e-5 and du0_rel <= 1e-5
    parity = all_max(0.0 if ok else 1.0) == 0.0
    del Us, Ss, Lam
    # entry mode "maps" (slice envelopes and slice maps all-gathered): the same bits, and its time
    Um, Sm_, _ = tshard.tshard_forward(Is, u0, ops, comm, entry_mode="maps")
    maps_ok = all_max(0.0 if (torch.equal(Um.view(torch.int32), U1s.view(torch.int32)) and
                              torch.equal(Sm_.view(torch.int32), S1s.view(torch.int32))) else 1.0) == 0.0
    del Um, Sm_, U1s, S1s, dI1
    Iqm = Is.clone().requires_grad_(True)

    def step_maps():
        Iqm.grad = None
        S_ = tshard.lif_tshard(Iqm, u0, beta=BETA, ops=ops, comm=comm, entry_mode="maps")
        torch.autograd.backward(S_, GSs)
    for _ in range(2):
        step_maps()
    ms_maps = all_max(event_ms(step_maps, 5))
    del Iqm

    Iqs = Is.clone().requires_grad_(True)

    def step_ts():
        Iqs.grad = None
        S_ = tshard.lif_tshard(Iqs, u0, beta=BETA, ops=ops, comm=comm)
        torch.autograd.backward(S_, GSs)
    for _ in range(max(args.warmup, 3)):
        step_ts()
    ms_ts = all_max(event_ms(step_ts, max(min(args.steps, 20), 5)))
    # one more step through the protocol with CUDA-event marks per phase
    tl = []
    U_, _, entry_ = tshard.tshard_forward(Is, u0, ops, comm, timeline=tl)
    tshard.tshard_backward(Is, entry_, U_, GSs, ops, comm, BETA, timeline=tl)
    torch.cuda.synchronize(dev)
    mine = [(tl[i][0], tl[i - 1][1].elapsed_time(tl[i][1])) for i in range(1, len(tl))]
    every = [None] * ws
    dist.all_gather_object(every, mine)
    per_phase = {}
    for lst in every:
        for name, v in lst:
            per_phase[name] = round(max(per_phase.get(name, 0.0), v), 4)
    del U_, entry_, Iqs
    torch.cuda.empty_cache()
    return parity, {
        "workload": C4_WORKLOAD, "path": "lif_tshard (entry_mode='speculate') fwd + autograd backward",
        "ranks": ws, "ms_per_step": ms_ts, "value": T * N / (ms_ts / 1e3), "unit": UNIT,
        "one_gpu_ms_per_step": ms1, "one_gpu_path": "lif_tuned(mode='scan') over the whole sequence, on each rank",
        "strong_scaling_efficiency": ms1 / (ws * ms_ts),
        "parity": {"U_S_bit_exact": ok, "dI_rel": dI_rel, "du0_rel": du0_rel,
                   "repair_rounds": info.get("repair_rounds")},
        "phases_ms_max_over_ranks": per_phase,
        "entry_mode_maps": {"ms_per_step": ms_maps, "strong_scaling_efficiency": ms1 / (ws * ms_maps),
                            "U_S_bit_exact": maps_ok,
                            "note": "slice envelopes and slice maps all-gathered, entry from the maps"},
        "note": "every rank holds the whole sequence for the check; the timed step moves only its slice"}


def c3_network(args, ws, rank, dev, clock=None):
    """Config 3: one training step (forward, backward, Adam) of the 700-256-256-20
    LIF network, B = 64 per GPU, T = 1024, beta = 0.9, Kaiming-uniform init,
    leaky readout, cross-entropy over 20 random labels, synthetic Bernoulli
    raster (rates U(0.5%, 4%)).  Data parallel: one bucketed all-reduce of the
    weight gradients per step when ws > 1 (the process group must exist).  The
    headline runs both LIF layers as spike-input layers (producer="spike": the
    input's spike mask, the fused Linear -> LIF forward over the active inputs,
    the sparse weight and bias gradients); the same step with nn.Linear then
    lif_tuned (producer="linear") is timed beside, and the two forwards'
    spikes are compared bit for bit.  The raster (183 MB) is larger than L2.
    Returns the record (rank 0's view; timings are maxima over ranks)."""
    import torch
    import torch.distributed as dist
    import torch.nn as nn

    from hard_resets_compose_b200 import _lib
    from hard_resets_compose_b200.shdnet import Net, synthetic_batch

    lib = _lib.load()
    T, B, H = 1024, 64, 256
    x, y = synthetic_batch(T, B, seed=1000 + rank, device=dev)
    stream = torch.cuda.current_stream(dev)

    def make(producer):
        torch.manual_seed(0)
        net = Net(mode="scan", beta=0.9, H=H, init="kaiming", readout="leaky", producer=producer).to(dev)
        # torch's fused Adam (one kernel per step, graph-capturable), in both arms
        opt = torch.optim.Adam(net.parameters(), lr=1e-3, capturable=True, fused=True)
        params = list(net.parameters())

        def fwd_bwd():
            loss = nn.functional.cross_entropy(net(x)[0], y)
            loss.backward()
            return loss

        with torch.no_grad():
            spikes = [s.clone() for s in net(x)[1]]
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                opt.zero_grad(set_to_none=True)
                fwd_bwd()
                opt.step()
        stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        opt.zero_grad(set_to_none=True)
        g_fb = torch.cuda.CUDAGraph()
        n0 = lib.lifb_kernel_launches()
        with torch.cuda.graph(g_fb):
            fwd_bwd()
        launches = lib.lifb_kernel_launches() - n0
        g_opt = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g_opt):
            opt.step()
        flat = torch.empty(sum(p.numel() for p in params), device=dev)

        def step():
            g_fb.replay()
            if ws > 1:  # data parallel: average the weight gradients (about 1 MB)
                torch.cat([p.grad.reshape(-1) for p in params], out=flat)
                dist.all_reduce(flat)
                flat.div_(ws)
                o = 0
                for p in params:
                    p.grad.copy_(flat[o:o + p.numel()].view_as(p.grad))
                    o += p.numel()
            g_opt.replay()
        # the graphs hold raw pointers into the net's parameters and the
        # optimizer's state: both must live as long as the graphs do
        return step, launches, spikes, (g_fb, g_opt, net, opt)

    def time_steps(step, steps):
        for _ in range(max(args.warmup, 3)):
            step()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)
        for a, b in evs:
            a.record(stream)
            step()
            b.record(stream)
        torch.cuda.synchronize(dev)
        ms = sum(a.elapsed_time(b) for a, b in evs) / len(evs)
        if ws > 1:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
            dist.barrier()
        return ms

    step_s, launches, spikes_s, keep_s = make("spike")
    step_l, _, spikes_l, keep_l = make("linear")
    same = torch.tensor([float(all(torch.equal(a, b) for a, b in zip(spikes_s, spikes_l)))], device=dev)
    if ws > 1:
        dist.all_reduce(same, op=dist.ReduceOp.MIN)
    if clock is not None:
        with clock:
            ms = time_steps(step_s, args.steps)
    else:
        ms = time_steps(step_s, args.steps)
    ms_linear = time_steps(step_l, max(args.steps // 2, 3))
    units = 2 * B * H * T * ws  # LIF neuron-steps per step, both layers, all ranks
    del keep_s, keep_l
    return {
        "metric": C3_METRIC, "ms_per_step": ms, "value": units / (ms / 1e3), "unit": UNIT,
        "producer": "spike (input spike mask, fused Linear -> LIF forward, sparse weight/bias gradient: "
                    "lifb_spike_mask, lifb_spike_linear_lif_fwd, lifb_spike_linear_wgrad)",
        "linear_producer": {"ms_per_step": ms_linear, "value": units / (ms_linear / 1e3),
                            "note": "the same step with nn.Linear then lif_tuned in both LIF layers"},
        "speedup_over_linear_producer": ms_linear / ms,
        "spikes_bit_equal_between_producers": bool(same.item() == 1.0),
        "gpu_launches_per_step": launches,
        "parallelism": f"data-parallel x{ws}, gradient all-reduce per step",
    }


def run_network(args, ws, rank, local):
    """`--workload c3`: the config-3 network step (c3_network) as its own line."""
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    clk = ClockSampler(local)
    rec = c3_network(args, ws, rank, dev, clock=clk)
    if rank == 0:
        print(json.dumps({
            "metric": C3_METRIC,
            "value": rec["value"], "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": rec["ms_per_step"], "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic Bernoulli raster, rates U(0.5%, 4%), 20 labels",
            "config": {"workload": "c3: network training step (forward, backward, Adam)", "beta": 0.9,
                       "init": "kaiming-uniform", "readout": "leaky (non-spiking integrator, mean over T)",
                       "lif_mode": "scan", "batch_per_gpu": 64, "seq_len": 1024, "producer": rec["producer"],
                       "parallelism": rec["parallelism"],
                       "step": "forward+backward and Adam (torch's fused Adam) each captured in a CUDA graph",
                       "l2": "the input raster (183 MB) and every layer tensor (64 MB) exceed or fill L2"},
            "linear_producer": rec["linear_producer"],
            "spikes_bit_equal_between_producers": rec["spikes_bit_equal_between_producers"],
            "gpu_launches": rec["gpu_launches_per_step"] * args.steps, "clocks": clk.record()}), flush=True)
    if ws > 1:
        dist.destroy_process_group()


def main():
    args = parse()
    ws, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, ws, rank)
        return
    if args.workload == "c1":
        run_c1(args, ws, rank, local)
        return
    if args.workload == "c3":
        run_network(args, ws, rank, local)
        return
    if args.workload == "c4":
        run_long(args, ws, rank, local)
        return
    if args.workload == "c5":
        run_sweep(args, ws, rank, local)
        return
    if args.workload in ("soft", "affine", "alif"):
        run_reset_family(args, ws, rank, local, args.workload)
        return

    import torch
    import torch.distributed as dist

    from hard_resets_compose_b200 import _lib
    from hard_resets_compose_b200 import lifscan as L

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    lib = _lib.load()

    def barrier():
        if ws > 1:
            dist.barrier()

    def max_over_ranks(x):
        if ws == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    numa_node = bind_numa(torch, dev)
    T, N = T_STEPS, N_PER_GPU
    g = torch.Generator().manual_seed(1000 + rank)
    I_h = (MU + SD * torch.randn(T, N, generator=g)).float()
    GS_h = torch.randn(T, N, generator=g).float()
    u0_h = torch.zeros(N)
    I = I_h.to(dev)
    GS = GS_h.to(dev)
    u0 = u0_h.to(dev)
    Iq = I.clone().requires_grad_(True)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    evict = torch.ones(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    sink = torch.empty((), dtype=torch.float32, device=dev)

    def flush_l2():
        # write a buffer larger than L2, then read another one so the written
        # lines are evicted (written back) here, outside the timed region:
        # every timed call starts with a cold L2 holding no dirty lines.
        flush.fill_(1.0)
        torch.sum(evict, dim=0, out=sink)
    stream = torch.cuda.current_stream(dev)

    def step():
        Iq.grad = None
        S = L.lif_tuned(Iq, u0, beta=BETA, theta=1.0, u_r=0.0, alpha=4.0, mode=args.mode) if args.mode != "auto" \
            else L.lif_auto(Iq, u0, beta=BETA)
        torch.autograd.backward(S, GS)
        return S

    def timed(fn, steps, launches_per_call=None):
        """Per-step CUDA events on the launching stream, L2 flushed between
        steps outside the events; returns (mean ms, kernel launches).  For a
        graph replay the library's launch counter does not move, so the
        launches recorded at capture time are used."""
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        barrier()
        torch.cuda.synchronize(dev)
        n0 = lib.lifb_kernel_launches()
        for a, b in evs:
            flush_l2()
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize(dev)
        n1 = lib.lifb_kernel_launches()
        barrier()
        ms = [a.elapsed_time(b) for a, b in evs]
        n = (n1 - n0) if launches_per_call is None else launches_per_call * steps
        return sum(ms) / len(ms), n

    def graphed(fn):
        """Capture fn (warmed up on a side stream) in a CUDA graph; returns
        (replay callable, kernel launches of this library per replay)."""
        side = torch.cuda.Stream(dev)
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            for _ in range(3):
                fn()
        stream.wait_stream(side)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        n0 = lib.lifb_kernel_launches()
        with torch.cuda.graph(g):
            fn()
        n1 = lib.lifb_kernel_launches()
        torch.cuda.synchronize(dev)
        return g.replay, n1 - n0

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize(dev)
    units = N * T * ws

    # eager: the autograd call as a training loop issues it, host overhead included
    ms_eager, _ = timed(step, args.steps)
    ms_eager = max_over_ranks(ms_eager)
    # the same step captured once in a CUDA graph, each replay timed alone
    # after an L2 flush (the event pair also holds the launch's latency)
    replay_step, per_step_launches = graphed(step)
    for _ in range(max(args.warmup, 3)):
        replay_step()
    ms_isolated, _ = timed(replay_step, args.steps, per_step_launches)
    ms_isolated = max_over_ranks(ms_isolated)
    # the headline: steps back to back over a ring of input sets larger than
    # L2 (each step's I and GS last touched C2_RING - 1 steps earlier, with
    # more than L2's capacity of other traffic since), one event pair
    ring_sets = [(I.clone().requires_grad_(True), torch.randn(T, N, generator=torch.Generator(device=dev).manual_seed(
        2000 + 10 * rank + r), device=dev)) for r in range(C2_RING - 1)]
    ring_sets.insert(0, (Iq, GS))

    def ring_step(Ir, Gr):
        def f():
            Ir.grad = None
            S_ = L.lif_tuned(Ir, u0, beta=BETA, theta=1.0, u_r=0.0, alpha=4.0, mode=args.mode) \
                if args.mode != "auto" else L.lif_auto(Ir, u0, beta=BETA)
            torch.autograd.backward(S_, Gr)
        return f
    ring = RingTimer(torch, dev, stream, lib, [ring_step(Ir, Gr) for Ir, Gr in ring_sets], barrier)
    with ClockSampler(local) as clk:
        ms_local = ring.ms_per_step(args.steps)
    launches = ring.launches_per_step * args.steps
    ms = max_over_ranks(ms_local)
    value = units / (ms / 1e3)

    # forward-only and per-call timings (roofline of the dominant call): the
    # calls lif_tuned itself makes for this shape and mode
    vpath = L._single_pass(T, N, args.mode) and args.mode != "auto"
    bwd_bytes = BWD_BYTES_V if vpath else BWD_BYTES

    def fwd_call():
        if vpath:
            return L.serial_forward_v(I, BETA, 1.0, 0.0, u0)
        return L.scan_forward_auto(I, BETA, 1.0, 0.0, u0) if args.mode == "scan" else \
            L.serial_forward_auto(I, BETA, 1.0, 0.0, u0)
    U, S = fwd_call()

    def bwd_call():  # exactly lif_tuned's backward call (S recomputed, GU zero)
        if vpath:
            return L.lif_backward_v(U, GS, BETA, 1.0, 4.0, C=T if args.mode == "serial" else L.scan_chunk_bwd(T, N))
        if args.mode == "scan":
            return L.scan_backward_auto(I, u0, U, None, GS, None, BETA, 1.0, 0.0, 4.0)
        return L.serial_backward_auto(I, u0, U, None, GS, None, BETA, 1.0, 0.0, 4.0)
    for _ in range(3):
        fwd_call()
        bwd_call()
    # per call, back to back over the same ring (forward: I of each set;
    # backward: that set's forward output and GS)
    fwd_sets = [(Ir.detach(),) for Ir, _ in ring_sets]
    bwd_sets = []
    for (Ir,), (_, Gr) in zip(fwd_sets, ring_sets):
        V_, _ = (L.serial_forward_v(Ir, BETA, 1.0, 0.0, u0) if vpath else
                 L.scan_forward_auto(Ir, BETA, 1.0, 0.0, u0))
        bwd_sets.append((Ir, V_, Gr))

    def fwd_of(Ir):
        if vpath:
            return lambda: L.serial_forward_v(Ir, BETA, 1.0, 0.0, u0)
        return (lambda: L.scan_forward_auto(Ir, BETA, 1.0, 0.0, u0)) if args.mode == "scan" else \
            (lambda: L.serial_forward_auto(Ir, BETA, 1.0, 0.0, u0))

    def bwd_of(Ir, Ur, Gr):
        if vpath:
            return lambda: L.lif_backward_v(Ur, Gr, BETA, 1.0, 4.0, C=T if args.mode == "serial" else
                                            L.scan_chunk_bwd(T, N))
        if args.mode == "scan":
            return lambda: L.scan_backward_auto(Ir, u0, Ur, None, Gr, None, BETA, 1.0, 0.0, 4.0)
        return lambda: L.serial_backward_auto(Ir, u0, Ur, None, Gr, None, BETA, 1.0, 0.0, 4.0)
    rf = RingTimer(torch, dev, stream, lib, [fwd_of(*a) for a in fwd_sets], barrier)
    rb = RingTimer(torch, dev, stream, lib, [bwd_of(*a) for a in bwd_sets], barrier)
    n_fwd, n_bwd = rf.launches_per_step, rb.launches_per_step
    ms_fwd = max_over_ranks(rf.ms_per_step(args.steps))
    ms_bwd = max_over_ranks(rb.ms_per_step(args.steps))
    del rf, rb, bwd_sets, fwd_sets
    hbm, peak_kind = peaks()
    per_call = {
        "fwd": {"ms": ms_fwd, "bytes": FWD_BYTES * N * T, "launches": n_fwd},
        "bwd": {"ms": ms_bwd, "bytes": bwd_bytes * N * T, "launches": n_bwd},
    }
    for v in per_call.values():
        v["gbs"] = v["bytes"] / (v["ms"] / 1e3) / 1e9
        v["frac"] = v["gbs"] / hbm
    dom = "fwd" if ms_fwd >= ms_bwd else "bwd"
    kname = {"fwd": f"lifb forward ({args.mode})", "bwd": f"lifb backward ({args.mode})"}[dom]
    tpu = traffic_per_unit(f"{args.mode}_{dom}" + ("_v" if vpath else ""))
    roofline = {
        "bound": "hbm", "kernel": kname, "launches_per_call": per_call[dom]["launches"],
        "achieved": per_call[dom]["gbs"], "peak": hbm, "peak_source": peak_kind, "unit": "GB/s",
        "frac": per_call[dom]["frac"],
        "traffic": (tpu * N * T) if tpu is not None else None,
        "algorithmic_bytes": per_call[dom]["bytes"],
        "step_frac": ((FWD_BYTES + bwd_bytes) * N * T) / (ms_local / 1e3) / 1e9 / hbm,
        "step_bytes_per_neuron_step": FWD_BYTES + bwd_bytes,
    }

    # end to end through the public API with host buffers: lif_tuned_host
    # (C-ABI lifb_lif_fwd_bwd_host_rows) takes pinned host I, GS, u0 and returns
    # host S, dI, du0; its H2D copies, kernels and D2H copies are all inside
    # the timed region.  The unpipelined eager equivalent is reported beside.
    e2e = None
    if not args.no_e2e:
        I_pin = I_h.pin_memory()
        GS_pin = GS_h.pin_memory()
        u0_pin = u0_h.pin_memory()
        host_out = (torch.empty(T, N).pin_memory(), torch.empty(T, N).pin_memory(), torch.empty(N).pin_memory())

        def e2e_host():
            L.lif_tuned_host(I_pin, GS_pin, u0_pin, beta=BETA, out=host_out)
        for _ in range(3):
            e2e_host()
        ms_e2e_host, _ = timed(e2e_host, max(args.steps // 2, 5))
        ms_e2e_host = max_over_ranks(ms_e2e_host)
        I_p = I_h.pin_memory()
        GS_p = GS_h.pin_memory()
        S_p = torch.empty(T, N).pin_memory()
        dI_p = torch.empty(T, N).pin_memory()
        du0_p = torch.empty(N).pin_memory()
        u0r = u0.clone().requires_grad_(True)

        def e2e_step():
            Id = I_p.to(dev, non_blocking=True).requires_grad_(True)
            G = GS_p.to(dev, non_blocking=True)
            u0r.grad = None
            S_ = L.lif_tuned(Id, u0r, beta=BETA, mode=args.mode) if args.mode != "auto" else \
                L.lif_auto(Id, u0r, beta=BETA)
            torch.autograd.backward(S_, G)
            S_p.copy_(S_.detach(), non_blocking=True)
            dI_p.copy_(Id.grad, non_blocking=True)
            du0_p.copy_(u0r.grad, non_blocking=True)
        for _ in range(3):
            e2e_step()
        ms_e2e, _ = timed(e2e_step, max(args.steps // 2, 5))
        ms_e2e = max_over_ranks(ms_e2e)
        # the copy floor: the same bytes moved with nothing else, on all
        # ranks at once (H2D of I and GS on one stream while S and dI come
        # back on another, and the same copies one after the other)
        dbuf = [torch.empty(T, N, device=dev) for _ in range(4)]
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)

        def copies(concurrent):
            s_in.wait_stream(stream)
            s_out.wait_stream(stream)
            so = s_out if concurrent else s_in
            with torch.cuda.stream(s_in):
                dbuf[0].copy_(I_pin, non_blocking=True)
                dbuf[1].copy_(GS_pin, non_blocking=True)
            with torch.cuda.stream(so):
                host_out[0].copy_(dbuf[2], non_blocking=True)
                host_out[1].copy_(dbuf[3], non_blocking=True)
            stream.wait_stream(s_in)
            stream.wait_stream(s_out)
        for _ in range(2):
            copies(True)
            copies(False)
        ms_floor, _ = timed(lambda: copies(True), max(args.steps // 2, 5))
        ms_floor = max_over_ranks(ms_floor)
        ms_floor_serial, _ = timed(lambda: copies(False), max(args.steps // 2, 5))
        ms_floor_serial = max_over_ranks(ms_floor_serial)
        del dbuf
        e2e = {"value": units / (ms_e2e_host / 1e3), "unit": UNIT, "ms_per_step": ms_e2e_host,
               "h2d_bytes_per_step": 2 * N * T * 4 + N * 4, "d2h_bytes_per_step": 2 * N * T * 4 + N * 4,
               "api": "lif_tuned_host (C-ABI lifb_lif_fwd_bwd_host_rows, blocks of time rows): pinned host I, GS, "
                      "u0 in; host S, dI, du0 out",
               "copy_floor_ms": ms_floor, "copy_floor_serial_ms": ms_floor_serial,
               "copy_floor_note": "the step's H2D (I, GS) and D2H (S, dI) bytes alone between the same pinned host "
                                  "buffers and the device, every rank at once; concurrent: H2D and D2H on two "
                                  "streams; serial: one after the other",
               "numa_node": numa_node,
               "unpipelined": {"value": units / (ms_e2e / 1e3), "ms_per_step": ms_e2e,
                               "api": "tensor.to(cuda) + lif_tuned + autograd.backward + copies back"}}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        v, threads, sample = cpu_oracle_rate(T, N, args.cpu_seconds)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}

    tshard_parity, c4_ts = None, None
    if ws > 1 and not args.no_tshard:
        tshard_parity, c4_ts = c4_time_sharded(args, ws, rank, dev, lib)
    c3 = None
    if not args.no_c3:
        c3_args = argparse.Namespace(**{**vars(args), "steps": 10, "warmup": 3})
        c3 = c3_network(c3_args, ws, rank, dev)
        c3["steps"] = c3_args.steps

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": max(args.warmup, 3), "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded torch.Generator, config 2 shape)",
            "config": {"workload": "c2: lif_tuned fwd+bwd, B*N=16384 per GPU, T=1024, beta=0.99, x~N(0.05,0.2^2)",
                       "mode": args.mode, "global_neurons": N * ws, "seq_len": T,
                       "parallelism": f"batch-sharded x{ws}, no collective",
                       "step": "lif_tuned forward + torch.autograd.backward; one CUDA graph holds one step per "
                               "input set of the ring",
                       "l2": f"inputs larger than L2: the steps run back to back over a ring of {C2_RING} input sets "
                             f"(I, GS: 128 MiB per set, 320 MiB touched per step), one event pair around all of "
                             f"them; isolated_step: each graph replay alone after an L2 flush (256 MiB written, "
                             f"then 256 MiB read), its own event pair"},
            "isolated_step": {"ms_per_step": ms_isolated, "value": units / (ms_isolated / 1e3)},
            "eager": {"ms_per_step": ms_eager, "value": units / (ms_eager / 1e3),
                      "note": "same step issued eagerly from Python each time after an L2 flush "
                              "(host overhead included)"},
            "fwd": {"ms": ms_fwd, "value": units / (ms_fwd / 1e3), "gbs": per_call["fwd"]["gbs"],
                    "frac": per_call["fwd"]["frac"]},
            "bwd": {"ms": ms_bwd, "value": units / (ms_bwd / 1e3), "gbs": per_call["bwd"]["gbs"],
                    "frac": per_call["bwd"]["frac"]},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": launches,
            "clocks": clk.record(),
        }
        if ws > 1 and not args.no_tshard:
            line["tshard_parity"] = tshard_parity
            line["c4_tshard"] = c4_ts
        if c3 is not None:
            line["c3"] = c3
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
