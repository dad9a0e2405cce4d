"""Shared test helpers: seeded CPU inputs (the reference's generator,
tests/test_fast.py:7-9) and comparison utilities."""
import numpy as np
import torch

from oracle import oracle as O


def gen(T, N, mu, sd, seed=0, u0_sd=0.0, grad=False):
    return O.gen_inputs(T, N, mu, sd, seed=seed, u0_sd=u0_sd, grad=grad)


def to_dev(dev, *arrays):
    return tuple(None if a is None else torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in arrays)


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    nb = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (nb if nb > 0 else 1.0))


def assert_bit_equal(got, want, what):
    got = np.asarray(got)
    want = np.asarray(want)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    # the reference's own criterion is torch.equal (elementwise ==); require bit equality here
    bad = got.view(np.uint32) != want.view(np.uint32)
    if bad.any():
        idx = np.argwhere(bad)[:5]
        raise AssertionError(f"{what}: {int(bad.sum())} elements differ, first at {idx.tolist()}: "
                             f"{got[tuple(idx[0])]!r} vs {want[tuple(idx[0])]!r}")
