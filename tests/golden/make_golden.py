"""Generate the golden fixtures that pin the CPU oracle to the reference.

Run once in a container that has the reference checked out (read-only) at
$LIFSCAN_REF (default: a directory named `reference` beside this repository):

    python tests/golden/make_golden.py

It imports the reference's own code:
  * lifscan/fast.py (PyTorch CPU): serial_forward_nograd (fast.py:69-81) and
    serial_backward (fast.py:227-239) -> the bit-exact forward anchor and the
    gradient anchor;
  * lifscan/triton_lif.py under TRITON_INTERPRET=1 (its Triton kernels run on
    the CPU through the interpreter, with numpy fp32 arithmetic and no FMA
    contraction): the v3 phases env_chunk/env_carry/build3/carry2
    (triton_lif.py:698-779, 578-606), scan_forward_v3 (:782), the v4 phases
    compose_group/carry_inner (:828-932), scan_forward_v4 (:935) and
    scan_backward_tiled (:512), including their internal map arrays and stats;
  * the soft-reset model: triton_lif.soft_serial_forward / soft_serial_backward
    (:1035-1082) and triton_soft.soft_scan_forward (interval maps, interpreted)
    and soft_adjoint_fft (float64 FFT) -> tests/golden/soft_*.npz
    (`--soft-only` regenerates just these);
  * the affine-reset model: triton_affine.aff_serial_forward /
    aff_scan_forward (interpreted) and LIFAffineFn's gradients (PyTorch CPU)
    over the (gamma, delta) x beta grid of tests/test_affine.py ->
    tests/golden/affine_grid.npz (`--affine-only`);
  * the ALIF model: triton_alif.alif_serial_forward (plain and tiled),
    alif_scan_forward with warm-up predictions, alif_warm_predict and
    alif_backward (serial and scan; interpreted), and ALIFFn's gradients, over
    the neuron classes of tests/test_alif.py -> tests/golden/alif_grid.npz
    (`--alif-only`);
  * near-threshold stress inputs (the method of experiments/e2b_stress.py,
    plus exact fp32 ties v == theta): fast.py's serial forward and its pruned
    scan with repair, and the Triton scan_forward_v3 / v4 with repair and their
    stats (interpreted) -> tests/golden/stress_near_threshold.npz
    (`--stress-only`).

Inputs are drawn on the CPU with torch.Generator (tests/test_fast.py:7-9) and
stored in the fixture too.  The GPU box never runs this script; the tests read
only the .npz files it writes next to itself.
"""
import os
import sys

os.environ["TRITON_INTERPRET"] = "1"
REF = os.environ.get("LIFSCAN_REF", os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "..",
                                                   "reference"))
sys.path.insert(0, REF)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import triton  # noqa: E402

from lifscan import fast  # noqa: E402
from lifscan import triton_lif as L  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def gen(T, N, mu, sd, seed, u0_sd):
    g = torch.Generator().manual_seed(seed)
    I = (mu + sd * torch.randn(T, N, generator=g)).to(torch.float32).contiguous()
    u0 = (u0_sd * torch.randn(N, generator=g)).to(torch.float32) if u0_sd else torch.zeros(N)
    GS = torch.randn(T, N, generator=g).to(torch.float32)
    return I, u0.contiguous(), GS


def v3_internals(I, beta, theta, u_r, u0, C, K):
    """The phases of scan_forward_v3 (triton_lif.py:782-803), run one by one."""
    T, N = I.shape
    M = T // C
    BN, BNc, BNr, D = 32, 16, 32, 8
    EC = torch.empty(M, N); EA = torch.empty(M, N); EB = torch.empty(M, N)
    De = D if C % D == 0 else 1
    L.env_chunk_kernel[(M, triton.cdiv(N, BNr))](I, EC, EA, EB, N, C, beta, u_r, BN=BNr, D=De)
    Lo = torch.empty(M, N)
    L.env_carry_kernel[(triton.cdiv(N, BNc),)](u0, EC, EA, EB, Lo, N, M, 1e-5, BN=BNc)
    MA = torch.empty(M, N); MB = torch.empty(M, N)
    MX = torch.empty(M, K, N); MC = torch.empty(M, K, N)
    MN = torch.empty(M, N, dtype=torch.int32); OVF = torch.empty(M, N, dtype=torch.int32)
    L.build3_kernel[(M, triton.cdiv(N, BN))](I, Lo, u0, MA, MB, MX, MC, MN, OVF, N, C, beta, theta, u_r,
                                             K=K, BN=BN)
    Starts = torch.empty(M, N)
    L.carry2_kernel[(triton.cdiv(N, BNc),)](I, u0, MA, MB, MX, MC, MN, OVF, Starts, N, M, C,
                                            beta, theta, u_r, K=K, BN=BNc, STAGES=1)
    return dict(Lo=Lo, MA=MA, MB=MB, MX=MX, MC=MC, MN=MN, OVF=OVF, Starts=Starts)


def v4_internals(I, beta, theta, u_r, u0, C, G, K, K2, base):
    """compose_group + carry over supers + carry_inner (triton_lif.py:951-965)."""
    T, N = I.shape
    M = T // C
    M2 = M // G
    BNg, BNc = 16, 16
    SA = torch.empty(M2, N); SB = torch.empty(M2, N)
    SX = torch.empty(M2, K2, N); SC = torch.empty(M2, K2, N)
    SN = torch.empty(M2, N, dtype=torch.int32); SOVF = torch.empty(M2, N, dtype=torch.int32)
    L.compose_group_kernel[(M2, triton.cdiv(N, BNg))](base["MA"], base["MB"], base["MX"], base["MC"],
                                                      base["MN"], base["OVF"], base["Lo"], u0,
                                                      SA, SB, SX, SC, SN, SOVF, N, G, theta, u_r,
                                                      K=K, K2=K2, BN=BNg)
    SStarts = torch.empty(M2, N)
    L.carry2_kernel[(triton.cdiv(N, BNc),)](I, u0, SA, SB, SX, SC, SN, SOVF, SStarts, N, M2, C * G,
                                            beta, theta, u_r, K=K2, BN=BNc, STAGES=1)
    Starts = torch.empty(M, N)
    L.carry_inner_kernel[(M2, triton.cdiv(N, BNc))](I, SStarts, base["MA"], base["MB"], base["MX"],
                                                    base["MC"], base["MN"], base["OVF"], Starts, N, G, C,
                                                    beta, theta, u_r, K=K, BN=BNc)
    return dict(SA=SA, SB=SB, SX=SX, SC=SC, SN=SN, SOVF=SOVF, SStarts=SStarts, Starts4=Starts)


FWD_CASES = [
    # name, T, N, mu, sd, seed, u0_sd, beta, u_r, C, K
    ("c1like", 512, 40, 0.1, 0.3, 0, 0.0, 0.9, 0.0, 64, 16),
    ("c2like", 512, 33, 0.05, 0.2, 1, 0.0, 0.99, 0.0, 64, 16),
    ("b05_neg", 256, 24, -0.1, 0.6, 2, 0.3, 0.5, -0.1, 32, 4),
    ("b1_ovf", 256, 24, 0.4, 0.2, 3, 0.3, 1.0, -0.1, 64, 2),
    ("b099_k64", 256, 17, 0.15, 0.4, 4, 0.3, 0.99, -0.1, 32, 64),
]

V4_CASES = [
    # name, T, N, mu, sd, seed, u0_sd, beta, u_r, C, G, K, K2
    ("v4a", 1024, 20, 0.15, 0.4, 5, 0.3, 0.99, -0.1, 32, 8, 8, 16),
    ("v4b", 512, 20, 0.1, 0.3, 6, 0.0, 0.9, 0.0, 16, 4, 4, 8),
]

BWD_CASES = [
    # name, T, N, mu, sd, seed, u0_sd, beta, u_r, alpha, detach, C
    ("bwd_det", 256, 24, 0.15, 0.4, 7, 0.2, 0.9, -0.1, 4.0, True, 32),
    ("bwd_nodet", 256, 24, 0.15, 0.4, 8, 0.2, 0.9, -0.1, 4.0, False, 64),
    ("bwd_c2like", 256, 33, 0.05, 0.2, 9, 0.0, 0.99, 0.0, 4.0, True, 64),
]


def npy(d):
    return {k: v.numpy() if torch.is_tensor(v) else np.asarray(v) for k, v in d.items()}


# soft reset: name, T, N, mu, sd, seed, u0_sd, beta, alpha, C, K
SOFT_CASES = [
    ("soft_b095", 512, 33, 0.15, 0.4, 5, 0.3, 0.95, 4.0, 32, 16),
    ("soft_b099", 1024, 16, 0.4, 0.3, 6, 0.3, 0.99, 4.0, 32, 32),
    ("soft_neg", 512, 24, -0.1, 0.6, 7, 0.3, 0.9, 2.0, 16, 16),
]


def soft_cases():
    """The soft-reset model (lifscan/triton_lif.py:1035-1082, lifscan/triton_soft.py):
    serial forward and exact interval-map scan (Triton interpreter), the fp32 serial
    adjoint (Triton interpreter) and the float64 FFT adjoint (PyTorch CPU)."""
    from lifscan import triton_soft as TS
    theta = 1.0
    for (name, T, N, mu, sd, seed, u0_sd, beta, alpha, C, K) in SOFT_CASES:
        I, u0, GS = gen(T, N, mu, sd, seed, u0_sd)
        U, S = L.soft_serial_forward(I, beta, theta, u0)
        st = {}
        U2, S2 = TS.soft_scan_forward(I, beta, theta, u0, C=C, K=K, repair=10 ** 6, stats=st)
        assert torch.equal(U2, U) and torch.equal(S2, S), name
        lam_serial = L.soft_serial_backward(I, u0, U, GS, beta, theta, alpha)
        uprev = torch.cat([u0[None], U[:-1]], 0)
        V = beta * uprev + I  # as LIFSoftScanFn forms it (lifscan/fit.py:138-139)
        lam_fft = TS.soft_adjoint_fft(V, GS, beta, theta, alpha)
        out = dict(I=I, u0=u0, GS=GS, U=U, S=S, V=V, Lam_serial=lam_serial, Lam_fft=lam_fft,
                   params=np.array([beta, theta, alpha, C, K], np.float64),
                   stats_keys=np.array(sorted(st)), stats_vals=np.array([st[k] for k in sorted(st)], np.float64))
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **npy(out))
        rel = ((lam_serial - lam_fft).norm() / lam_fft.norm()).item()
        print(name, st, "serial vs fft rel", rel)


# affine reset: the (gamma, delta) x beta grid of tests/test_affine.py:7-9 at
# reduced size (T, N), C = 32, K = 16
AFF_GRID = ((0.0, 0.0), (0.0, -0.2), (0.3, -0.1), (0.7, -0.5), (1.0, -1.0), (0.5, 0.2))
AFF_BETAS = (0.9, 0.97)
AFF_T, AFF_N, AFF_C, AFF_K = 256, 16, 32, 16


def affine_cases():
    """The affine-reset model (lifscan/triton_affine.py): serial forward and the
    exact piecewise-affine map scan (Triton interpreter), and LIFAffineFn's
    gradients for I, u0, beta, gamma, delta (PyTorch CPU, its own backward)."""
    from lifscan import triton_affine as A
    theta, alpha = 1.0, 4.0
    out = {}
    for gi, (gamma, delta) in enumerate(AFF_GRID):
        for bi, beta in enumerate(AFF_BETAS):
            key = f"g{gi}b{bi}"
            I, u0, GS = gen(AFF_T, AFF_N, 0.15, 0.4, 20 + 2 * gi + bi, 0.2)
            U, S = A.aff_serial_forward(I, beta, theta, gamma, delta, u0)
            st = {}
            U2, S2 = A.aff_scan_forward(I, beta, theta, gamma, delta, u0, C=AFF_C, K=AFF_K, repair=10 ** 6,
                                        stats=st)
            assert torch.equal(U2, U) and torch.equal(S2, S), key
            Ig = I.clone().requires_grad_(True)
            ug = u0.clone().requires_grad_(True)
            ps = [torch.tensor(v, dtype=torch.float32, requires_grad=True) for v in (beta, gamma, delta)]
            Sg = A.lif_affine(Ig, ug, ps[0], ps[1], ps[2], theta=theta, alpha=alpha, mode="serial")
            assert torch.equal(Sg.detach(), S), key
            (GS * Sg).sum().backward()
            out.update({f"{key}_I": I, f"{key}_u0": u0, f"{key}_GS": GS, f"{key}_U": U, f"{key}_S": S,
                        f"{key}_dI": Ig.grad, f"{key}_du0": ug.grad,
                        f"{key}_dp": torch.stack([p.grad for p in ps]),
                        f"{key}_params": np.array([beta, theta, gamma, delta, alpha], np.float64),
                        f"{key}_stats": np.array([st["repair_iters"], st["overflow_frac"], st["mean_pieces"]])})
            print(key, gamma, delta, beta, st, "spikes", float(S.mean()))
    np.savez_compressed(os.path.join(HERE, "affine_grid.npz"), **npy(out))


# ALIF: the neuron classes of tests/test_alif.py:10 (name, beta, rho, q) x free
# membrane drive m (:11) at reduced size (T, N), chunks of C = 32 rows
ALIF_CASES = (("lsnn", 0.95, 0.995, 0.9), ("glif2", 0.99, 0.96, 0.2), ("appD-a", 0.9, 0.95, 0.5))
ALIF_M = (0.5, 2.0)
ALIF_T, ALIF_N, ALIF_C = 512, 8, 32


def alif_cases():
    """The ALIF model (lifscan/triton_alif.py): serial forward (plain and
    time-tiled), the exact box scan with warm-up predictions (repair to
    convergence), alif_warm_predict, the serial and two-level scan adjoints
    (Triton interpreter), and ALIFFn's gradients for I, u0, w0, beta, rho, q,
    theta0 (its own backward, PyTorch CPU + interpreter)."""
    import math
    from lifscan import triton_alif as A
    theta0, u_r, alpha = 1.0, 0.0, 4.0
    out = {}
    for ci, (name, beta, rho, q) in enumerate(ALIF_CASES):
        for mi, mfree in enumerate(ALIF_M):
            key = f"a{ci}m{mi}"
            g = torch.Generator().manual_seed(40 + 2 * ci + mi)
            I = ((1 - beta) * mfree + 0.5 * math.sqrt(1 - beta * beta)
                 * torch.randn(ALIF_T, ALIF_N, generator=g)).contiguous()
            u0 = torch.zeros(ALIF_N)
            w0 = (0.1 * torch.rand(ALIF_N, generator=g)).contiguous()
            GS = torch.randn(ALIF_T, ALIF_N, generator=g)
            U, W, S = A.alif_serial_forward(I, beta, rho, q, theta0, u_r, u0, w0)
            Ut, Wt, St = A.alif_serial_forward(I, beta, rho, q, theta0, u_r, u0, w0, D=8)
            assert torch.equal(Ut, U) and torch.equal(Wt, W) and torch.equal(St, S), key
            WP = A.alif_warm_predict(I, beta, rho, q, theta0, u_r, u0, w0, ALIF_C, Wn=4)
            st = {}
            U2, W2, S2 = A.alif_scan_forward(I, beta, rho, q, theta0, u_r, u0, w0, WP.contiguous(), 0.1 * q,
                                             C=ALIF_C, K1=16, K2=32, repair=10 ** 6, stats=st)
            assert torch.equal(U2, U) and torch.equal(W2, W) and torch.equal(S2, S), key
            LV, LW = A.alif_backward(I, U, W, S, GS, beta, rho, q, theta0, u0, w0, alpha=alpha, mode="serial")
            LVs, LWs = A.alif_backward(I, U, W, S, GS, beta, rho, q, theta0, u0, w0, alpha=alpha, mode="scan",
                                       C=ALIF_C)
            # the reference's two-level scan adjoint agrees with its serial sweep
            assert ((LVs - LV).norm() / LV.norm()).item() < 1e-5, key
            assert ((LWs - LW).norm() / LW.norm()).item() < 1e-5, key
            Ig = I.clone().requires_grad_(True)
            ug = u0.clone().requires_grad_(True)
            wg = w0.clone().requires_grad_(True)
            ps = [torch.tensor(v, dtype=torch.float32, requires_grad=True) for v in (beta, rho, q, theta0)]
            Sg, _, _ = A.alif(Ig, ug, wg, ps[0], ps[1], ps[2], ps[3], u_r=u_r, alpha=alpha, fwd="serial",
                              bwd="serial")
            assert torch.equal(Sg.detach(), S), key
            (GS * Sg).sum().backward()
            out.update({f"{key}_I": I, f"{key}_u0": u0, f"{key}_w0": w0, f"{key}_GS": GS, f"{key}_U": U,
                        f"{key}_W": W, f"{key}_S": S, f"{key}_WP": WP, f"{key}_LV": LV, f"{key}_LW": LW,
                        f"{key}_dI": Ig.grad, f"{key}_du0": ug.grad,
                        f"{key}_dw0": wg.grad, f"{key}_dp": torch.stack([p.grad for p in ps]),
                        f"{key}_params": np.array([beta, rho, q, theta0, u_r, alpha], np.float64),
                        f"{key}_stats": np.array([st["repair_iters"], st["miss_frac"], st["mean_pieces"]])})
            print(key, name, mfree, st, "spikes", float(S.mean()), flush=True)
    np.savez_compressed(os.path.join(HERE, "alif_grid.npz"), **npy(out))


def stress_inputs(T, N, beta, eps, p_hit, seed, tie32=False):
    """Near-threshold stress inputs for theta = 1, u_r = 0, u0 = 0.  The drive
    is x ~ N(0.15, 0.4^2).  With probability p_hit per (t, n) x_t is replaced:
      tie32=False (experiments/e2b_stress.py:10-17): in float64, by the value
        that puts the float64 serial pre-reset potential within +-eps of
        theta; the fp32 copy then lands within an ulp or two of it;
      tie32=True: in fp32, by theta - fl(beta*u), so that the fp32 serial
        potential fl(fl(beta*u) + x) equals theta exactly wherever that
        difference is exact (a spike decided by >= alone)."""
    g = torch.Generator().manual_seed(seed)
    dt = torch.float32 if tie32 else torch.float64
    I = (0.15 + 0.4 * torch.randn(T, N, dtype=torch.float64, generator=g)).to(dt)
    hit = torch.rand(T, N, generator=g) < p_hit
    u = torch.zeros(N, dtype=dt)
    for t in range(T):
        if tie32:
            tgt = torch.ones(N, dtype=dt) - beta * u  # fp32: fl(1 - fl(beta*u))
        else:
            tgt = 1.0 + eps * (2 * torch.rand(N, dtype=dt, generator=g) - 1) - beta * u
        I[t] = torch.where(hit[t], tgt, I[t])
        v = beta * u + I[t]
        u = torch.where(v >= 1.0, torch.zeros_like(v), v)
    return I.to(torch.float32).contiguous()


STRESS_CASES = [  # name, T, N, beta, eps, p_hit, seed, tie32
    ("b09_e1e-6", 512, 32, 0.9, 1e-6, 0.3, 31, False),
    ("b099_e1e-7", 512, 32, 0.99, 1e-7, 0.3, 32, False),
    ("b099_tie", 512, 32, 0.99, 0.0, 0.3, 33, True),
    ("b09_tie", 512, 32, 0.9, 0.0, 0.3, 34, True),
]


def stress_cases():
    theta, u_r = 1.0, 0.0
    out = {}
    for (name, T, N, beta, eps, p_hit, seed, tie32) in STRESS_CASES:
        I = stress_inputs(T, N, beta, eps, p_hit, seed, tie32)
        u0 = torch.zeros(N)
        us, ss, vs = fast.serial_forward_nograd(I, beta, theta, u_r, u0)
        stp = {}
        Up, Sp = fast.scan_forward_pruned(I, beta, theta, u_r, u0, C=64, K=64, repair=10 ** 6, stats=stp)[:2]
        assert torch.equal(Up, us) and torch.equal(Sp, ss), name
        st3, st4 = {}, {}
        U3, S3 = L.scan_forward_v3(I, beta, theta, u_r, u0, C=64, K=16, repair=10 ** 6, stats=st3)
        U4, S4 = L.scan_forward_v4(I, beta, theta, u_r, u0, C=32, G=4, K=16, K2=32, repair=10 ** 6, stats=st4)
        assert torch.equal(U3, us) and torch.equal(S3, ss) and torch.equal(U4, us) and torch.equal(S4, ss), name
        ties = int((vs == theta).sum())
        out.update({f"{name}_I": I, f"{name}_U": us, f"{name}_S": ss,
                    f"{name}_params": np.array([beta, theta, u_r], np.float64),
                    f"{name}_v3_keys": np.array(sorted(st3)),
                    f"{name}_v3_vals": np.array([st3[k] for k in sorted(st3)], np.float64),
                    f"{name}_v4_keys": np.array(sorted(st4)),
                    f"{name}_v4_vals": np.array([st4[k] for k in sorted(st4)], np.float64),
                    f"{name}_ties": np.array(ties)})
        print(name, "exact ties", ties, "v3", st3, "v4", st4, "pruned repair", stp.get("repair_iters"))
    np.savez_compressed(os.path.join(HERE, "stress_near_threshold.npz"), **npy(out))


def main():
    theta = 1.0
    if "--stress-only" in sys.argv:
        stress_cases()
        return
    if "--alif-only" in sys.argv:
        alif_cases()
        return
    if "--soft-only" in sys.argv:
        soft_cases()
        return
    if "--affine-only" in sys.argv:
        affine_cases()
        return
    soft_cases()
    affine_cases()
    alif_cases()
    stress_cases()
    for (name, T, N, mu, sd, seed, u0_sd, beta, u_r, C, K) in FWD_CASES:
        I, u0, _ = gen(T, N, mu, sd, seed, u0_sd)
        us, ss, vs = fast.serial_forward_nograd(I, beta, theta, u_r, u0)
        inter = v3_internals(I, beta, theta, u_r, u0, C, K)
        st0, st = {}, {}
        U0, S0 = L.scan_forward_v3(I, beta, theta, u_r, u0, C=C, K=K, repair=0, stats=st0)
        U, S = L.scan_forward_v3(I, beta, theta, u_r, u0, C=C, K=K, repair=10 ** 6, stats=st)
        assert torch.equal(U, us) and torch.equal(S, ss), name
        out = dict(I=I, u0=u0, U=us, S=ss, U_norepair=U0, S_norepair=S0,
                   params=np.array([beta, theta, u_r, C, K], np.float64),
                   stats_keys=np.array(sorted(st)), stats_vals=np.array([st[k] for k in sorted(st)], np.float64),
                   stats0_vals=np.array([st0[k] for k in sorted(st0)], np.float64))
        out.update(inter)
        np.savez_compressed(os.path.join(HERE, f"fwd_{name}.npz"), **npy(out))
        print(name, st, st0)

    for (name, T, N, mu, sd, seed, u0_sd, beta, u_r, C, G, K, K2) in V4_CASES:
        I, u0, _ = gen(T, N, mu, sd, seed, u0_sd)
        us, ss, _ = fast.serial_forward_nograd(I, beta, theta, u_r, u0)
        base = v3_internals(I, beta, theta, u_r, u0, C, K)
        inter = v4_internals(I, beta, theta, u_r, u0, C, G, K, K2, base)
        st = {}
        U, S = L.scan_forward_v4(I, beta, theta, u_r, u0, C=C, G=G, K=K, K2=K2, repair=10 ** 6, stats=st)
        assert torch.equal(U, us) and torch.equal(S, ss), name
        out = dict(I=I, u0=u0, U=us, S=ss, params=np.array([beta, theta, u_r, C, G, K, K2], np.float64),
                   stats_keys=np.array(sorted(st)), stats_vals=np.array([st[k] for k in sorted(st)], np.float64))
        out.update({k: base[k] for k in ("Lo", "MN", "OVF", "MA", "MB")})
        out.update(inter)
        np.savez_compressed(os.path.join(HERE, f"v4_{name}.npz"), **npy(out))
        print(name, st)

    for (name, T, N, mu, sd, seed, u0_sd, beta, u_r, alpha, detach, C) in BWD_CASES:
        I, u0, GS = gen(T, N, mu, sd, seed, u0_sd)
        GU = torch.randn(T, N, generator=torch.Generator().manual_seed(seed + 100)) if not detach \
            else torch.zeros(T, N)
        us, ss, vs = fast.serial_forward_nograd(I, beta, theta, u_r, u0)
        lam_fast = fast.serial_backward(vs, ss, GS, GU, beta, theta, u_r, alpha, detach_reset=detach)
        lam_tri = L.scan_backward_tiled(I, u0, us, ss, GS, GU, beta, theta, u_r, alpha, detach=detach,
                                        C=C, BNr=16, D=4)
        # fp64 autograd through the reference's differentiable serial loop (fast.py:52-66)
        Id = I.double().requires_grad_(True)
        u0d = u0.double().requires_grad_(True)
        ud, sd_ = fast.serial_lif(Id, beta, theta, u_r, u0d, alpha=alpha, detach_reset=detach)
        ((GS.double() * sd_).sum() + (GU.double() * ud).sum()).backward()
        out = dict(I=I, u0=u0, U=us, S=ss, GS=GS, GU=GU, Lam_fast=lam_fast, Lam_triton=lam_tri,
                   dI_fp64=Id.grad, du0_fp64=u0d.grad,
                   params=np.array([beta, theta, u_r, alpha, float(detach), C], np.float64))
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **npy(out))
        rel = ((lam_fast - lam_tri).norm() / lam_fast.norm()).item()
        print(name, "fast vs triton-interp rel", rel)


if __name__ == "__main__":
    main()
