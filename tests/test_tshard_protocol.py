"""Host protocol of the time-sharded scan on CPU: ranks as gloo processes
(world size 2 and 4) and as threads (2 to 8 ranks), with the oracle standing in for the
per-slice GPU phases (tests/tshard_oracle_ops.py).  The slices' U and S must
equal the serial recurrence over the whole sequence bit for bit, and the
gradients its adjoint within 1e-5, whatever the entry guesses were; a rank
that drops out makes the others fail instead of hang."""
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O
from tests.helpers import assert_bit_equal, gen, rel
from tests.tshard_oracle_ops import OracleSliceOps

CASES = {
    # name: (T_total, N, mu, sd, beta)
    "spiking": (3072, 48, 0.15, 0.4, 0.9),
    "c4like": (3072, 32, 0.02, 0.1, 0.99),
    "rare": (1536, 32, -0.01, 0.05, 1.0),  # random walk, few spikes: errors carry across slices
}


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _slice_run(comm, case, mode, info, K=8, K3=32):
    """mode: "maps" (oracle slice maps), "corrupt" (maps that guess 0.5),
    "speculate" (no maps: segments after the first from lead-ins, the last
    one's end handed on as the next slice's entry guess) or
    "speculate_leadin" (the same with a separate lead-in pass for the guess);
    K, K3: chunk and slice map capacities."""
    from hard_resets_compose_b200 import tshard
    T_total, N, mu, sd, beta = CASES[case]
    I, u0, GS = gen(T_total, N, mu, sd, seed=3, u0_sd=0.3, grad=True)
    a, b = tshard.slice_rows(T_total, comm.world, comm.rank)
    ops_mode = {"corrupt": "corrupt", "speculate_leadin": "no_tail"}.get(mode, "maps")
    ops = OracleSliceOps(b - a, N, beta, 1.0, 0.0, C=64, K=K, K3=K3, mode=ops_mode)
    It, u0t, Gt = (torch.from_numpy(np.ascontiguousarray(x)) for x in (I[a:b], u0, GS[a:b]))
    U, S, entry = tshard.tshard_forward(It, u0t, ops, comm, info=info,
                                        entry_mode="speculate" if mode.startswith("speculate") else "maps")
    Lam, du0 = tshard.tshard_backward(It, entry, U, Gt, ops, comm, beta)
    return U.numpy(), S.numpy(), Lam.numpy(), du0.numpy()


def _check(case, world, results):
    T_total, N, mu, sd, beta = CASES[case]
    I, u0, GS = gen(T_total, N, mu, sd, seed=3, u0_sd=0.3, grad=True)
    Us, Ss = O.serial_forward(I, beta, 1.0, 0.0, u0)
    Lref = O.serial_backward(I, u0, Us, Ss, GS, None, beta, 1.0, 0.0, 4.0, True)
    U = np.concatenate([r[0] for r in results])
    S = np.concatenate([r[1] for r in results])
    Lam = np.concatenate([r[2] for r in results])
    assert_bit_equal(U, Us, "U")
    assert_bit_equal(S, Ss, "S")
    assert rel(Lam, Lref) < 1e-5
    assert rel(results[0][3], beta * Lref[0]) < 1e-5
    for r in results[1:]:
        assert not r[3].any()


@pytest.mark.parametrize("mode", ("maps", "corrupt", "speculate", "speculate_leadin"))
@pytest.mark.parametrize("case", sorted(CASES))
@pytest.mark.parametrize("world", (2, 3, 4, 6, 8))
def test_protocol_threads(case, mode, world):
    from hard_resets_compose_b200 import tshard
    infos = [dict() for _ in range(world)]
    res = tshard.run_local(world, lambda c: _slice_run(c, case, mode, infos[c.rank]))
    _check(case, world, res)
    rounds = infos[0]["repair_rounds"]
    assert all(i["repair_rounds"] == rounds for i in infos)  # same collective steps on every rank
    assert rounds <= world - 1
    if mode == "corrupt" and case == "rare" and world == 4:
        assert rounds >= 2  # the wrong guesses reach across more than one slice


def _gloo_worker(rank, world, port, case, mode, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        from hard_resets_compose_b200 import tshard
        info = {}
        U, S, Lam, du0 = _slice_run(tshard.TorchComm(), case, mode, info)
        np.savez(os.path.join(out_dir, f"r{rank}.npz"), U=U, S=S, Lam=Lam, du0=du0,
                 rounds=info["repair_rounds"])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,case,mode", ((2, "spiking", "maps"), (4, "c4like", "maps"), (4, "rare", "corrupt"),
                                             (4, "c4like", "speculate")))
def test_protocol_gloo(tmp_path, world, case, mode):
    mp.spawn(_gloo_worker, args=(world, _free_port(), case, mode, str(tmp_path)), nprocs=world, join=True)
    res = []
    for r in range(world):
        z = np.load(tmp_path / f"r{r}.npz")
        res.append((z["U"], z["S"], z["Lam"], z["du0"]))
        assert int(z["rounds"]) == int(np.load(tmp_path / "r0.npz")["rounds"])
    _check(case, world, res)


def _dropout_worker(rank, world, port, out_dir):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        return  # leaves before the first exchange, without any collective in flight
    from hard_resets_compose_b200 import tshard
    try:
        _slice_run(tshard.TorchComm(), "spiking", "maps", {})
        outcome = "finished"
    except Exception as e:  # noqa: BLE001 - the outcome is what the test checks
        outcome = "error: " + type(e).__name__
    with open(os.path.join(out_dir, "r0.txt"), "w") as f:
        f.write(outcome)


def test_rank_dropout_fails_fast(tmp_path):
    """A rank that never joins the envelope exchange: the other rank's
    all-gather ends with an error within the process-group timeout."""
    mp.spawn(_dropout_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    outcome = (tmp_path / "r0.txt").read_text()
    assert outcome.startswith("error"), outcome


def test_thread_rank_failure_propagates():
    from hard_resets_compose_b200 import tshard

    def fn(comm):
        if comm.rank == 2:
            raise RuntimeError("rank 2 failed")
        return _slice_run(comm, "spiking", "maps", {})

    with pytest.raises(RuntimeError, match="rank 2 failed"):
        tshard.run_local(3, fn)


class _LateComm:
    """A comm whose rank enters every exchange `delay` seconds late (a slow
    rank, injected on the host)."""

    def __init__(self, comm, delay):
        self.comm, self.delay = comm, delay
        self.world, self.rank = comm.world, comm.rank

    def all_gather(self, t):
        time.sleep(self.delay)
        return self.comm.all_gather(t)

    def shift(self, t):
        time.sleep(self.delay)
        return self.comm.shift(t)


@pytest.mark.parametrize("mode", ("maps", "speculate"))
def test_slow_rank_changes_nothing(mode):
    """One rank reaches every exchange late: the others wait for it at the
    collective, and the result is the same bits."""
    from hard_resets_compose_b200 import tshard
    world = 4
    res = tshard.run_local(world, lambda c: _slice_run(_LateComm(c, 0.05 if c.rank == 2 else 0.0), "c4like",
                                                       mode, {}))
    _check("c4like", world, res)


@pytest.mark.parametrize("world", (2, 4))
@pytest.mark.parametrize("case", sorted(CASES))
def test_overflowing_maps_stay_exact(case, world):
    """Chunk and slice maps of capacity 1 overflow almost everywhere; an
    overflowed slice map is only a worse entry guess, which the repair rounds
    correct."""
    from hard_resets_compose_b200 import tshard
    infos = [dict() for _ in range(world)]
    res = tshard.run_local(world, lambda c: _slice_run(c, case, "maps", infos[c.rank], K=1, K3=1))
    _check(case, world, res)
    assert infos[0]["repair_rounds"] <= world - 1
