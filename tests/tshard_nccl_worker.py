"""One rank of the time-sharded scan over NCCL (launched by torchrun from
tests/test_gpu_tshard.py): rank r takes rows [r*T, (r+1)*T) of a seeded
sequence, runs lif_tshard forward and backward on cuda:r and saves U, S, dI
and du0 for the test to compare with the oracle."""
import argparse
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

from oracle import oracle as O  # noqa: E402  (input generator only)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--T", type=int, required=True)
    ap.add_argument("--N", type=int, required=True)
    ap.add_argument("--mu", type=float, default=0.02)
    ap.add_argument("--sd", type=float, default=0.1)
    ap.add_argument("--beta", type=float, default=0.99)
    ap.add_argument("--out", required=True)
    a = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        from hard_resets_compose_b200 import tshard
        I, u0, GS = O.gen_inputs(a.T, a.N, a.mu, a.sd, seed=0, grad=True)
        s0, s1 = tshard.slice_rows(a.T, world, rank)
        It = torch.from_numpy(np.ascontiguousarray(I[s0:s1])).to(dev).requires_grad_(True)
        u0t = torch.from_numpy(u0).to(dev).requires_grad_(True)
        Gt = torch.from_numpy(np.ascontiguousarray(GS[s0:s1])).to(dev)
        S = tshard.lif_tshard(It, u0t, beta=a.beta)
        (S * Gt).sum().backward()
        torch.cuda.synchronize()
        np.savez(os.path.join(a.out, f"r{rank}.npz"), S=S.detach().cpu().numpy(), dI=It.grad.cpu().numpy(),
                 du0=u0t.grad.cpu().numpy())
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
