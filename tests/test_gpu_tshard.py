"""Time-sharded scan on the GPU (lifb_tshard_* through the C ABI).

Ranks are emulated as threads on one GPU (tshard.run_local) for the parity
grid, and run as one process per GPU over NCCL when the box has two or more
GPUs.  The slices together must equal the oracle's serial recurrence over
the whole sequence bit for bit, and the adjoint within 1e-5 (config 4's
inputs at reduced T, plus regimes with many, few and no spikes)."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_bit_equal, gen, rel

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(cuda, T_total, N, mu, sd, beta, world, u_r=0.0, u0_sd=0.0, K3=64, seed=0, entry_mode="maps"):
    from hard_resets_compose_b200 import tshard
    I, u0, GS = gen(T_total, N, mu, sd, seed=seed, u0_sd=u0_sd, grad=True)
    Id = torch.from_numpy(I).to(cuda)
    Gd = torch.from_numpy(GS).to(cuda)
    u0d = torch.from_numpy(u0).to(cuda)
    T = T_total // world
    infos = [dict() for _ in range(world)]

    def rank_fn(comm):
        r = comm.rank
        ops = tshard.CudaSliceOps(T, N, cuda, beta, 1.0, u_r, K3=K3)
        Ir = Id[r * T:(r + 1) * T]
        U, S, entry = tshard.tshard_forward(Ir, u0d, ops, comm, info=infos[r], entry_mode=entry_mode)
        Lam, du0 = tshard.tshard_backward(Ir, entry, U, Gd[r * T:(r + 1) * T], ops, comm, beta)
        return U, S, Lam, du0

    res = tshard.run_local(world, rank_fn)
    torch.cuda.synchronize()
    Us, Ss = O.serial_forward(I, beta, 1.0, u_r, u0)
    Lref = O.serial_backward(I, u0, Us, Ss, GS, None, beta, 1.0, u_r, 4.0, True)
    U = torch.cat([r[0] for r in res]).cpu().numpy()
    S = torch.cat([r[1] for r in res]).cpu().numpy()
    Lam = torch.cat([r[2] for r in res]).cpu().numpy()
    assert_bit_equal(S, Ss, "S")
    assert_bit_equal(U, Us, "U")
    assert rel(Lam, Lref) < 1e-5
    assert rel(res[0][3].cpu().numpy(), beta * Lref[0]) < 1e-5
    return infos


@pytest.mark.parametrize("entry_mode", ("maps", "speculate"))
@pytest.mark.parametrize("world", (2, 4, 8))
@pytest.mark.parametrize("beta,mu,sd", ((0.99, 0.02, 0.1), (0.9, 0.15, 0.4), (1.0, -0.01, 0.05), (0.5, 0.4, 0.2)))
def test_tshard_threads_bit_exact(cuda, world, beta, mu, sd, entry_mode):
    infos = _run(cuda, 1 << 15, 1024, mu, sd, beta, world, u0_sd=0.3, entry_mode=entry_mode)
    assert infos[0]["repair_rounds"] <= world - 1


def test_tshard_overflowing_slice_maps(cuda):
    """K3 = 1: the slice maps overflow, the entries are guesses and the
    cross-slice repair makes the result exact."""
    _run(cuda, 1 << 15, 1024, 0.15, 0.4, 0.9, 4, u_r=-0.1, u0_sd=0.3, K3=1)


@pytest.mark.parametrize("entry_mode", ("maps", "speculate"))
def test_tshard_c4_reduced(cuda, entry_mode):
    """Config 4's distribution and width at T = 2^18 over 4 slices (slices of
    2^16 rows: the speculative mode runs segments with lead-ins inside them)."""
    infos = _run(cuda, 1 << 18, 1024, 0.02, 0.1, 0.99, 4, entry_mode=entry_mode)
    assert infos[0]["repair_rounds"] <= 3


def test_tshard_nccl_two_gpus(tmp_path):
    """One process per GPU over NCCL (skipped on a one-GPU box)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    T, N = 1 << 16, 1024
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr=127.0.0.1", "--master-port=29531",
           os.path.join(ROOT, "tests", "tshard_nccl_worker.py"), "--T", str(T), "--N", str(N), "--out",
           str(tmp_path)]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    p = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-4000:]
    I, u0, GS = gen(T, N, 0.02, 0.1, seed=0, grad=True)
    Us, Ss = O.serial_forward(I, 0.99, 1.0, 0.0, u0)
    Lref = O.serial_backward(I, u0, Us, Ss, GS, None, 0.99, 1.0, 0.0, 4.0, True)
    z = [np.load(tmp_path / f"r{r}.npz") for r in range(2)]
    assert_bit_equal(np.concatenate([x["S"] for x in z]), Ss, "S")
    assert rel(np.concatenate([x["dI"] for x in z]), Lref) < 1e-5
    assert rel(z[0]["du0"] + z[1]["du0"], 0.99 * Lref[0]) < 1e-5
