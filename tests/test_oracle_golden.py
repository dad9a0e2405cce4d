"""Pin the CPU oracle to the reference (no GPU needed).

tests/golden/*.npz were written by tests/golden/make_golden.py from the
reference's own code: lifscan/fast.py (serial forward / backward) and the
reference's Triton kernels run through the Triton interpreter (v3/v4 phases,
maps, starts, stats and the tiled backward).  The oracle must reproduce the
integer/bit-level quantities exactly and the gradients to 1e-6 relative.
"""
import glob
import os

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import assert_bit_equal, rel

GOLD = os.path.join(os.path.dirname(__file__), "golden")
FWD = sorted(glob.glob(os.path.join(GOLD, "fwd_*.npz")))
V4 = sorted(glob.glob(os.path.join(GOLD, "v4_*.npz")))
BWD = sorted(glob.glob(os.path.join(GOLD, "bwd_*.npz")))


def _valid(arr, cnt, K):
    mask = np.arange(K)[None, :, None] < cnt[:, None, :]
    return np.where(mask, arr, 0.0).astype(np.float32)


def _stats(z):
    return {str(k): float(v) for k, v in zip(z["stats_keys"], z["stats_vals"])}


def test_fixtures_present():
    assert len(FWD) >= 5 and len(V4) >= 2 and len(BWD) >= 3


@pytest.mark.parametrize("path", FWD, ids=os.path.basename)
def test_serial_forward_matches_fast_py(path):
    z = np.load(path)
    beta, theta, u_r = (float(v) for v in z["params"][:3])
    U, S = O.serial_forward(z["I"], beta, theta, u_r, z["u0"])
    assert_bit_equal(U, z["U"], "U")
    assert_bit_equal(S, z["S"], "S")


@pytest.mark.parametrize("path", FWD, ids=os.path.basename)
def test_v3_phases_match_reference_kernels(path):
    z = np.load(path)
    beta, theta, u_r, C, K = z["params"]
    C, K = int(C), int(K)
    I, u0 = z["I"], z["u0"]
    Lo = O.envelope(I, u0, C, float(beta), float(u_r))
    assert_bit_equal(Lo, z["Lo"], "Lo (env_chunk + env_carry)")
    d = O.build_maps(I, u0, Lo, C, K, float(beta), float(theta), float(u_r))
    for k in ("MA", "MB", "MN", "OVF"):
        assert_bit_equal(d[k], z[k], k)
    assert_bit_equal(_valid(d["MX"], d["MN"], K), _valid(z["MX"], z["MN"], K), "MX (live slots)")
    assert_bit_equal(_valid(d["MC"], d["MN"], K), _valid(z["MC"], z["MN"], K), "MC (live slots)")


@pytest.mark.parametrize("path", FWD, ids=os.path.basename)
def test_v3_outputs_and_stats(path):
    z = np.load(path)
    beta, theta, u_r, C, K = z["params"]
    C, K = int(C), int(K)
    U, S, st = O.scan_forward_v3(z["I"], float(beta), float(theta), float(u_r), z["u0"], C=C, K=K)
    assert_bit_equal(U, z["U"], "U after repair")
    assert_bit_equal(S, z["S"], "S after repair")
    ref = _stats(z)
    assert st["repair_iters"] == int(ref["repair_iters"])
    assert st["max_pieces"] == int(ref["max_pieces"])
    assert abs(st["overflow_frac"] - ref["overflow_frac"]) < 1e-6
    assert abs(st["mean_pieces"] - ref["mean_pieces"]) < 1e-5
    # without repair the replay from the carried starts must match the reference's too
    U0, S0, _ = O.scan_forward_v3(z["I"], float(beta), float(theta), float(u_r), z["u0"], C=C, K=K, repair=0)
    assert_bit_equal(U0, z["U_norepair"], "U without repair")
    assert_bit_equal(S0, z["S_norepair"], "S without repair")


@pytest.mark.parametrize("path", V4, ids=os.path.basename)
def test_v4_phases_outputs_and_stats(path):
    z = np.load(path)
    beta, theta, u_r, C, G, K, K2 = z["params"]
    C, G, K, K2 = int(C), int(G), int(K), int(K2)
    U, S, st, d = O.scan_forward_v4(z["I"], float(beta), float(theta), float(u_r), z["u0"], C=C, G=G, K=K,
                                    K2=K2, return_internals=True)
    assert_bit_equal(U, z["U"], "U")
    assert_bit_equal(S, z["S"], "S")
    for k in ("SA", "SB", "SN", "SOVF", "SStarts"):
        assert_bit_equal(d[k], z[k], k)
    assert_bit_equal(_valid(d["SX"], d["SN"], K2), _valid(z["SX"], z["SN"], K2), "SX (live slots)")
    assert_bit_equal(_valid(d["SC"], d["SN"], K2), _valid(z["SC"], z["SN"], K2), "SC (live slots)")
    ref = _stats(z)
    assert st["repair_iters"] == int(ref["repair_iters"])
    assert st["super_max_pieces"] == int(ref["super_max_pieces"])
    for k in ("overflow_frac", "super_overflow_frac"):
        assert abs(st[k] - ref[k]) < 1e-6, k
    for k in ("mean_pieces", "super_mean_pieces"):
        assert abs(st[k] - ref[k]) < 1e-5, k


@pytest.mark.parametrize("path", V4, ids=os.path.basename)
def test_v4_carry_inner_matches_reference(path):
    z = np.load(path)
    beta, theta, u_r, C, G, K, K2 = z["params"]
    C, G, K, K2 = int(C), int(G), int(K), int(K2)
    # carry_inner's chunk starts are the replay starts before any repair round
    U, S, st, d = O.scan_forward_v4(z["I"], float(beta), float(theta), float(u_r), z["u0"], C=C, G=G, K=K,
                                    K2=K2, repair=0, return_internals=True)
    assert_bit_equal(d["Starts"], z["Starts4"], "chunk starts from carry_inner")


@pytest.mark.parametrize("path", BWD, ids=os.path.basename)
def test_backward_matches_reference(path):
    z = np.load(path)
    beta, theta, u_r, alpha, det, C = z["params"]
    det = bool(det)
    args = (z["I"], z["u0"], z["U"], z["S"], z["GS"], z["GU"], float(beta), float(theta), float(u_r), float(alpha),
            det)
    lam_serial = O.serial_backward(*args)
    lam_scan = O.scan_backward(*args, C=int(C))
    assert rel(lam_serial, z["Lam_fast"]) < 1e-6
    assert rel(lam_scan, z["Lam_triton"]) < 1e-6
    assert rel(lam_scan, z["Lam_fast"]) < 1e-6
    # and against fp64 autograd through the reference's differentiable serial loop
    assert rel(lam_serial, z["dI_fp64"]) < 1e-5
    assert rel(float(beta) * lam_serial[0], z["du0_fp64"]) < 1e-5


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "soft_*.npz"))), ids=os.path.basename)
def test_oracle_soft_reset_matches_reference(path):
    """Soft-reset model: the oracle's recurrence equals the reference's serial
    forward (and its exact interval-map scan) bit for bit; its adjoint matches
    the reference's fp32 serial adjoint and, in double, its float64 FFT adjoint."""
    z = np.load(path)
    beta, theta, alpha = (float(v) for v in z["params"][:3])
    U, S, V = O.soft_serial_forward(z["I"], beta, theta, z["u0"], want_v=True)
    assert_bit_equal(U, z["U"], "U")
    assert_bit_equal(S, z["S"], "S")
    assert_bit_equal(V, z["V"], "V")
    lam = O.soft_serial_backward(z["I"], z["u0"], U, z["GS"], beta, theta, alpha)
    lam_d = O.soft_serial_backward(z["I"], z["u0"], U, z["GS"], beta, theta, alpha, double=True)
    assert rel(lam, z["Lam_serial"]) < 1e-6
    assert rel(lam_d, z["Lam_fft"]) < 1e-6


AFF = os.path.join(GOLD, "affine_grid.npz")
AFF_KEYS = [f"g{g}b{b}" for g in range(6) for b in range(2)]


@pytest.mark.parametrize("key", AFF_KEYS)
def test_oracle_affine_reset_matches_reference(key):
    """Affine-reset model over the (gamma, delta) x beta grid of the
    reference's tests/test_affine.py: the oracle's recurrence equals the
    reference's serial forward (and its exact piecewise-affine map scan) bit
    for bit; its adjoint and (dbeta, dgamma, ddelta) match LIFAffineFn's own
    backward (Hillis-Steele scan in fp32, so within rounding)."""
    z = np.load(AFF)
    beta, theta, gamma, delta, alpha = (float(v) for v in z[f"{key}_params"])
    I, u0, GS = z[f"{key}_I"], z[f"{key}_u0"], z[f"{key}_GS"]
    U, S = O.aff_serial_forward(I, beta, theta, gamma, delta, u0)
    assert_bit_equal(U, z[f"{key}_U"], "U")
    assert_bit_equal(S, z[f"{key}_S"], "S")
    lam, pg = O.aff_serial_backward(I, u0, U, GS, beta, theta, gamma, alpha)
    lam_d, pg_d = O.aff_serial_backward(I, u0, U, GS, beta, theta, gamma, alpha, double=True)
    assert rel(lam, z[f"{key}_dI"]) < 1e-6
    assert rel(lam_d, z[f"{key}_dI"]) < 1e-6
    assert rel(beta * lam[0], z[f"{key}_du0"]) < 1e-6
    dp = z[f"{key}_dp"].astype(np.float64)
    for i in range(3):
        assert abs(pg[i] - dp[i]) <= 1e-5 * (abs(dp[i]) + 1e-3), (i, pg, dp)
        assert abs(pg_d[i] - dp[i]) <= 1e-5 * (abs(dp[i]) + 1e-3), (i, pg_d, dp)


def test_oracle_affine_contains_hard_and_soft():
    """gamma = 0, delta = u_r is the hard reset and gamma = 1, delta = -theta
    the soft reset, bit for bit (lifscan/triton_affine.py:1-4)."""
    rng = np.random.default_rng(3)
    I = (0.15 + 0.4 * rng.standard_normal((700, 13))).astype(np.float32)
    u0 = (0.3 * rng.standard_normal(13)).astype(np.float32)
    Ua, Sa = O.aff_serial_forward(I, 0.95, 1.0, 0.0, -0.2, u0)
    Uh, Sh = O.serial_forward(I, 0.95, 1.0, -0.2, u0)
    assert_bit_equal(Ua, Uh, "U hard")
    assert_bit_equal(Sa, Sh, "S hard")
    Ua, Sa = O.aff_serial_forward(I, 0.95, 1.0, 1.0, -1.0, u0)
    Us, Ss = O.soft_serial_forward(I, 0.95, 1.0, u0)
    assert_bit_equal(Ua, Us, "U soft")
    assert_bit_equal(Sa, Ss, "S soft")


ALIF = os.path.join(GOLD, "alif_grid.npz")
ALIF_KEYS = [f"a{c}m{m}" for c in range(3) for m in range(2)]


@pytest.mark.parametrize("key", ALIF_KEYS)
def test_oracle_alif_matches_reference(key):
    """ALIF over the neuron classes of the reference's tests/test_alif.py: the
    oracle's recurrence equals the reference's serial forward (and its exact
    box scan) bit for bit, its warm-up prediction equals alif_warm_predict,
    its adjoint pair matches the reference's serial sweep (which the
    generating script checked against its two-level scan), and its parameter
    sums match ALIFFn's own backward."""
    z = np.load(ALIF)
    beta, rho, q, theta0, u_r, alpha = (float(v) for v in z[f"{key}_params"])
    I, u0, w0, GS = (z[f"{key}_{k}"] for k in ("I", "u0", "w0", "GS"))
    U, W, S = O.alif_serial_forward(I, beta, rho, q, theta0, u_r, u0, w0)
    assert_bit_equal(U, z[f"{key}_U"], "U")
    assert_bit_equal(W, z[f"{key}_W"], "W")
    assert_bit_equal(S, z[f"{key}_S"], "S")
    WP = O.alif_warm_predict(I, beta, rho, q, theta0, u_r, u0, w0, 32, Wn=4)
    assert_bit_equal(WP, z[f"{key}_WP"], "WP")
    LV, LW, lwm1, pg = O.alif_serial_backward(I, u0, w0, U, W, S, GS, beta, rho, q, theta0, alpha)
    assert rel(LV, z[f"{key}_LV"]) < 1e-6
    assert rel(LW, z[f"{key}_LW"]) < 1e-6
    assert rel(LV, z[f"{key}_dI"]) < 1e-6
    assert rel(beta * LV[0], z[f"{key}_du0"]) < 1e-6
    assert rel(lwm1, z[f"{key}_dw0"]) < 1e-5
    dp = z[f"{key}_dp"].astype(np.float64)
    for i in range(4):
        assert abs(pg[i] - dp[i]) <= 1e-5 * (abs(dp[i]) + 1e-3), (i, pg, dp)


def test_oracle_alif_reduces_to_hard_reset():
    """q = 0 and w0 = 0 keep the adaptation at 0 (fl(rho*0) = 0), so ALIF is the
    hard reset with theta = theta0 bit for bit; and with q = 0, lw never enters
    lv's recurrence (d = gs), so lv is the hard reset's adjoint."""
    rng = np.random.default_rng(4)
    I = (0.12 + 0.4 * rng.standard_normal((600, 11))).astype(np.float32)
    u0 = (0.3 * rng.standard_normal(11)).astype(np.float32)
    w0 = np.zeros(11, np.float32)
    GS = rng.standard_normal((600, 11)).astype(np.float32)
    U, W, S = O.alif_serial_forward(I, 0.93, 0.97, 0.0, 1.0, -0.1, u0, w0)
    Uh, Sh = O.serial_forward(I, 0.93, 1.0, -0.1, u0)
    assert_bit_equal(U, Uh, "U")
    assert_bit_equal(S, Sh, "S")
    assert not W.any()
    LV, _, _, _ = O.alif_serial_backward(I, u0, w0, U, W, S, GS, 0.93, 0.97, 0.0, 1.0, 4.0)
    Lh = O.serial_backward(I, u0, Uh, Sh, GS, None, 0.93, 1.0, -0.1, 4.0, True)
    assert rel(LV, Lh) < 1e-6


def test_oracle_alif_warm_predict_from_row0_is_exact():
    """A warm-up that reaches row 0 starts from (u0, w0), so the prediction is
    the true entry adaptation (lifscan/triton_alif.py:78-79)."""
    rng = np.random.default_rng(5)
    T, N, C = 512, 6, 32
    I = (0.1 + 0.3 * rng.standard_normal((T, N))).astype(np.float32)
    u0 = np.zeros(N, np.float32)
    w0 = (0.1 * rng.random(N)).astype(np.float32)
    _, W, _ = O.alif_serial_forward(I, 0.95, 0.995, 0.9, 1.0, 0.0, u0, w0)
    WP = O.alif_warm_predict(I, 0.95, 0.995, 0.9, 1.0, 0.0, u0, w0, C, Wn=T // C)
    want = np.concatenate([w0[None], W[C - 1:-1:C]], 0)
    assert_bit_equal(WP, want, "WP")
