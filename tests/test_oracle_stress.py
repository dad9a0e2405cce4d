"""Pin the CPU oracle to the reference on near-threshold stress inputs (no GPU
needed).

tests/golden/stress_near_threshold.npz was written by
tests/golden/make_golden.py --stress-only from the reference's own code. Its
inputs follow experiments/e2b_stress.py: 30% of the steps land within 1e-6 or
1e-7 of theta in float64. Two further cases put the fp32 potential exactly on
theta, so that `v >= theta` alone decides the spike. The fixture holds the
reference's serial forward (lifscan/fast.py:69-81), which its pruned scan,
Triton scan_forward_v3 and scan_forward_v4 (with repair) all reproduce, and
the Triton scans' stats. The oracle must reproduce the outputs bit for bit and
the stats exactly.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import assert_bit_equal

GOLD = os.path.join(os.path.dirname(__file__), "golden", "stress_near_threshold.npz")
CASES = ["b09_e1e-6", "b099_e1e-7", "b099_tie", "b09_tie"]


def _case(name):
    z = np.load(GOLD)
    beta, theta, u_r = (float(v) for v in z[f"{name}_params"])
    return z, beta, theta, u_r


def _stats(z, name, level):
    return {str(k): float(v) for k, v in zip(z[f"{name}_{level}_keys"], z[f"{name}_{level}_vals"])}


def test_stress_inputs_reach_the_threshold():
    z = np.load(GOLD)
    for name in CASES:
        assert int(z[f"{name}_ties"]) > 200, name  # steps whose fp32 potential equals theta exactly


@pytest.mark.parametrize("name", CASES)
def test_stress_serial_forward(name):
    z, beta, theta, u_r = _case(name)
    I = z[f"{name}_I"]
    U, S = O.serial_forward(I, beta, theta, u_r, np.zeros(I.shape[1], np.float32))
    assert_bit_equal(U, z[f"{name}_U"], "U")
    assert_bit_equal(S, z[f"{name}_S"], "S")


@pytest.mark.parametrize("name", CASES)
def test_stress_v3(name):
    z, beta, theta, u_r = _case(name)
    I = z[f"{name}_I"]
    U, S, st = O.scan_forward_v3(I, beta, theta, u_r, np.zeros(I.shape[1], np.float32), C=64, K=16)
    assert_bit_equal(U, z[f"{name}_U"], "U")
    assert_bit_equal(S, z[f"{name}_S"], "S")
    ref = _stats(z, name, "v3")
    assert st["repair_iters"] == int(ref["repair_iters"])
    assert st["max_pieces"] == int(ref["max_pieces"])
    assert abs(st["overflow_frac"] - ref["overflow_frac"]) < 1e-6
    assert abs(st["mean_pieces"] - ref["mean_pieces"]) < 1e-5


@pytest.mark.parametrize("name", CASES)
def test_stress_v4(name):
    z, beta, theta, u_r = _case(name)
    I = z[f"{name}_I"]
    U, S, st = O.scan_forward_v4(I, beta, theta, u_r, np.zeros(I.shape[1], np.float32), C=32, G=4, K=16, K2=32)
    assert_bit_equal(U, z[f"{name}_U"], "U")
    assert_bit_equal(S, z[f"{name}_S"], "S")
    ref = _stats(z, name, "v4")
    assert st["repair_iters"] == int(ref["repair_iters"])
    assert st["super_max_pieces"] == int(ref["super_max_pieces"])
    for k in ("overflow_frac", "super_overflow_frac"):
        assert abs(st[k] - ref[k]) < 1e-6, k
    for k in ("mean_pieces", "super_mean_pieces"):
        assert abs(st[k] - ref[k]) < 1e-5, k
