"""Near-threshold stress inputs on the GPU, through the library (the fixture
of tests/golden/make_golden.py --stress-only, pinned to the reference's
fast.py and Triton scans by tests/test_oracle_stress.py). 30% of the steps
land within 1e-6 or 1e-7 of theta (experiments/e2b_stress.py), or exactly on it
in fp32. The serial forward, scan_forward_v3, scan_forward_v4 and
scan_forward_auto must reproduce the reference's spikes and potentials bit for
bit, and the v3/v4 stats must equal the reference's."""
import os

import numpy as np
import pytest

from tests.helpers import assert_bit_equal, to_dev

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden", "stress_near_threshold.npz")
CASES = ["b09_e1e-6", "b099_e1e-7", "b099_tie", "b09_tie"]


def L():
    from hard_resets_compose_b200 import lifscan
    return lifscan


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("name", CASES)
def test_stress_forward_paths(cuda, name):
    z = np.load(GOLD)
    beta, theta, u_r = (float(v) for v in z[f"{name}_params"])
    I = z[f"{name}_I"]
    Id, u0d = to_dev(cuda, I, np.zeros(I.shape[1], np.float32))
    for what, (U, S) in (("serial", L().serial_forward(Id, beta, theta, u_r, u0d)),
                         ("auto", L().scan_forward_auto(Id, beta, theta, u_r, u0d))):
        assert_bit_equal(_np(U), z[f"{name}_U"], f"{what} U")
        assert_bit_equal(_np(S), z[f"{name}_S"], f"{what} S")
    st3, st4 = {}, {}
    U, S = L().scan_forward_v3(Id, beta, theta, u_r, u0d, C=64, K=16, stats=st3)
    assert_bit_equal(_np(U), z[f"{name}_U"], "v3 U")
    assert_bit_equal(_np(S), z[f"{name}_S"], "v3 S")
    U, S = L().scan_forward_v4(Id, beta, theta, u_r, u0d, C=32, G=4, K=16, K2=32, stats=st4)
    assert_bit_equal(_np(U), z[f"{name}_U"], "v4 U")
    assert_bit_equal(_np(S), z[f"{name}_S"], "v4 S")
    for level, st in (("v3", st3), ("v4", st4)):
        ref = {str(k): float(v) for k, v in zip(z[f"{name}_{level}_keys"], z[f"{name}_{level}_vals"])}
        assert st["repair_iters"] == int(ref["repair_iters"]), level
        for k, v in ref.items():
            assert abs(st[k] - v) < 1e-5, (level, k, st[k], v)
