"""GPU backward and autograd parity through the C ABI.

Gradients must match the reference's backward within relative error 1e-5
(north star).  References: the oracle's restatement of
lifscan/fast.py:227-239 (serial adjoint) and of the tiled scan
(lifscan/triton_lif.py:512-526), the reference's own outputs stored in
tests/golden/bwd_*.npz, and fp64 autograd through fast.serial_lif."""
import glob
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_bit_equal, gen, rel, to_dev

pytestmark = pytest.mark.gpu
TOL = 1e-5  # relative (Frobenius) error bound on dI and du0
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def L():
    from hard_resets_compose_b200 import lifscan
    return lifscan


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLD, "bwd_*.npz"))), ids=os.path.basename)
def test_golden_reference_gradients(cuda, path):
    z = np.load(path)
    beta, theta, u_r, alpha, det, C = (float(v) for v in z["params"])
    det = bool(det)
    d = to_dev(cuda, z["I"], z["u0"], z["U"], z["S"], z["GS"], z["GU"])
    GU = d[5] if not det else None
    l1 = L().serial_backward(*d[:5], GU, beta, theta, u_r, alpha, det)
    l2 = L().scan_backward_tiled(*d[:5], GU, beta, theta, u_r, alpha, det, C=int(C))
    assert rel(_np(l1), z["Lam_fast"]) < TOL
    assert rel(_np(l2), z["Lam_fast"]) < TOL
    assert rel(_np(l2), z["Lam_triton"]) < TOL
    assert rel(_np(l1), z["dI_fp64"]) < TOL


@pytest.mark.parametrize("detach", (True, False))
@pytest.mark.parametrize("N,T,C", ((100, 4096, 64), (1000, 2048, 128), (5000, 1024, 64), (37, 512, 8)))
def test_backward_vs_oracle(cuda, detach, N, T, C):
    I, u0, GS = gen(T, N, 0.15, 0.4, seed=1, u0_sd=0.2, grad=True)
    U, S = O.serial_forward(I, 0.9, 1.0, -0.1, u0)
    GU = np.random.default_rng(2).standard_normal(I.shape).astype(np.float32)
    ref = O.serial_backward(I, u0, U, S, GS, GU, 0.9, 1.0, -0.1, 4.0, detach)
    d = to_dev(cuda, I, u0, U, S, GS, GU)
    l1 = L().serial_backward(*d, 0.9, 1.0, -0.1, 4.0, detach)
    l2 = L().scan_backward_tiled(*d, 0.9, 1.0, -0.1, 4.0, detach, C=C)
    assert rel(_np(l1), ref) < TOL
    assert rel(_np(l2), ref) < TOL


@pytest.mark.parametrize("mode", ("scan", "serial"))
def test_lif_tuned_c2_forward_backward(cuda, mode):
    """Config 2: lif_tuned fwd+bwd, B*N = 16384, T = 1024,
    x ~ N(0.05, 0.2^2), beta = 0.99, default surrogate, upstream grad N(0, 1)."""
    T, N, beta = 1024, 16384, 0.99
    I, u0, GS = gen(T, N, 0.05, 0.2, seed=0, grad=True)
    Us, Ss = O.serial_forward(I, beta, 1.0, 0.0, u0)
    dI_ref = O.serial_backward(I, u0, Us, Ss, GS, None, beta, 1.0, 0.0, 4.0, True)
    Id, u0d, GSd = to_dev(cuda, I, u0, GS)
    Id.requires_grad_(True)
    u0d.requires_grad_(True)
    S = L().lif_tuned(Id, u0d, beta=beta, mode=mode)
    (S * GSd).sum().backward()
    assert_bit_equal(_np(S), Ss, "S")
    assert rel(_np(Id.grad), dI_ref) < TOL
    assert rel(_np(u0d.grad), beta * dI_ref[0]) < TOL


def test_lif_auto_and_legacy_layer(cuda):
    T, N = 2048, 1000
    I, u0, GS = gen(T, N, 0.15, 0.4, seed=3, grad=True)
    Us, Ss = O.serial_forward(I, 0.9, 1.0, 0.0, u0)
    dI_ref = O.serial_backward(I, u0, Us, Ss, GS, None, 0.9, 1.0, 0.0, 4.0, True)
    for f in (lambda x, u: L().lif_auto(x, u, beta=0.9),
              lambda x, u: L().lif(x, u, beta=0.9, mode="scan", C=64),
              lambda x, u: L().lif(x, u, beta=0.9, mode="serial")):
        Id, u0d, GSd = to_dev(cuda, I, u0, GS)
        Id.requires_grad_(True)
        S = f(Id, u0d)
        (S * GSd).sum().backward()
        assert_bit_equal(_np(S), Ss, "S")
        assert rel(_np(Id.grad), dI_ref) < TOL


def test_gradient_against_fp64_autograd(cuda):
    """fp32 scan gradient vs an fp64 autograd pass through a plain serial
    recurrence in torch (the reference's fast.serial_lif, restated)."""
    T, N, beta, alpha = 512, 64, 0.9, 4.0
    I, u0, GS = gen(T, N, 0.15, 0.4, seed=4, grad=True)
    Ix = torch.from_numpy(I).double().requires_grad_(True)
    u = torch.zeros(N, dtype=torch.float64)
    ss = []
    for t in range(T):
        v = beta * u + Ix[t]
        sg = torch.sigmoid(alpha * (v - 1.0))
        # Heaviside forward, ds/dv = alpha*sg*(1-sg) backward (lifscan/fast.py:33-51)
        s = (v >= 1.0).double() + (sg - sg.detach())
        u = v * (1 - s.detach())  # detached reset to u_r = 0
        ss.append(s)
    (torch.from_numpy(GS).double() * torch.stack(ss)).sum().backward()
    Id, u0d, GSd = to_dev(cuda, I, u0, GS)
    Id.requires_grad_(True)
    S = L().lif_tuned(Id, u0d, beta=beta, mode="scan")
    (S * GSd).sum().backward()
    assert rel(_np(Id.grad), Ix.grad.numpy()) < 1e-5


@pytest.mark.parametrize("N,block_n", ((16384, 2048), (1000, 256), (4096, 4096), (16384, 1024), (777, 128)))
def test_lif_tuned_host_pipeline(cuda, N, block_n):
    """Host-buffer forward+backward (lifb_lif_fwd_bwd_host): spikes bit-exact,
    dI and du0 within 1e-5 of the oracle, for block counts that leave a
    ragged last block, a single block, and reuse of the staging slots."""
    T, beta = 1024, 0.99
    I, u0, GS = gen(T, N, 0.05, 0.2, seed=5, u0_sd=0.3, grad=True)
    Us, Ss = O.serial_forward(I, beta, 1.0, 0.0, u0)
    dI_ref = O.serial_backward(I, u0, Us, Ss, GS, None, beta, 1.0, 0.0, 4.0, True)
    It = torch.from_numpy(I).pin_memory()
    Gt = torch.from_numpy(GS).pin_memory()
    S, dI, du0 = L().lif_tuned_host(It, Gt, torch.from_numpy(u0), beta=beta, block_n=block_n)
    torch.cuda.synchronize()
    assert_bit_equal(S.numpy(), Ss, "S")
    assert rel(dI.numpy(), dI_ref) < TOL
    assert rel(du0.numpy(), beta * dI_ref[0]) < TOL
    # a second call reuses the library's copy streams and the staging slots
    S2, dI2, _ = L().lif_tuned_host(It, Gt, torch.from_numpy(u0), beta=beta, block_n=block_n)
    torch.cuda.synchronize()
    assert_bit_equal(S2.numpy(), Ss, "S (second call)")
    assert np.array_equal(dI2.numpy(), dI.numpy())


@pytest.mark.parametrize("N,T,block_t", ((16384, 1024, None), (1000, 1000, 96), (1024, 1024, 1024),
                                         (4096, 1024, 16), (512, 37, 5), (8, 64, 1)))
def test_lif_tuned_host_row_blocks(cuda, N, T, block_t):
    """Host-buffer forward+backward over blocks of time rows
    (lifb_lif_fwd_bwd_host_rows): spikes bit-exact, dI and du0 within 1e-5 of
    the oracle and bit-equal to the neuron-block pipeline, for a ragged last
    block, a single block, many blocks through four slots, and one-row blocks."""
    beta = 0.99
    I, u0, GS = gen(T, N, 0.05, 0.2, seed=11, u0_sd=0.3, grad=True)
    Us, Ss = O.serial_forward(I, beta, 1.0, 0.0, u0)
    dI_ref = O.serial_backward(I, u0, Us, Ss, GS, None, beta, 1.0, 0.0, 4.0, True)
    It = torch.from_numpy(I).pin_memory()
    Gt = torch.from_numpy(GS).pin_memory()
    S, dI, du0 = L().lif_tuned_host(It, Gt, torch.from_numpy(u0), beta=beta, block_t=block_t)
    assert_bit_equal(S.numpy(), Ss, "S")
    assert rel(dI.numpy(), dI_ref) < TOL
    assert rel(du0.numpy(), beta * dI_ref[0]) < TOL
    Sc, dIc, du0c = L().lif_tuned_host(It, Gt, torch.from_numpy(u0), beta=beta, block_n=max(4, N // 2 // 4 * 4))
    assert np.array_equal(dIc.numpy(), dI.numpy())
    assert np.array_equal(du0c.numpy(), du0.numpy())
    # a second call reuses the copy streams and the slots
    S2, dI2, _ = L().lif_tuned_host(It, Gt, torch.from_numpy(u0), beta=beta, block_t=block_t)
    assert_bit_equal(S2.numpy(), Ss, "S (second call)")
    assert np.array_equal(dI2.numpy(), dI.numpy())


def test_lif_tuned_host_row_blocks_refusals(cuda):
    from hard_resets_compose_b200 import _lib
    lib = _lib.load()
    z = torch.zeros(4, 6).pin_memory()
    with pytest.raises(ValueError):
        L().lif_tuned_host(z, z, block_t=2)  # N % 4 != 0: the neuron-block form only
    z4 = torch.zeros(4, 8).pin_memory()
    with pytest.raises(ValueError):
        L().lif_tuned_host(z4, z4, block_t=0)
    assert lib.lifb_lif_fwd_bwd_host_rows_block(1024, 16384) == 256
    assert lib.lifb_lif_fwd_bwd_host_rows_block(10, 16384) == 10
    assert lib.lifb_lif_fwd_bwd_host_rows_block(1024, 1 << 24) == 1


@pytest.mark.parametrize("beta", (0.5, 0.9, 0.99, 1.0))
@pytest.mark.parametrize("N,T,C", ((1000, 4096, 64), (1024, 1 << 16, 1024), (777, 2048, 128), (64, 4096, 4096)))
def test_scan_backward_fast_path(cuda, beta, N, T, C):
    """Detached reset: chunks replayed from lam_end = 0 plus the tail fix-up,
    with and without S supplied, against the oracle's serial adjoint."""
    I, u0, GS = gen(T, N, 0.05, 0.2, seed=13, u0_sd=0.3, grad=True)
    U, S = O.serial_forward(I, beta, 1.0, 0.0, u0)
    ref = O.serial_backward(I, u0, U, S, GS, None, beta, 1.0, 0.0, 4.0, True)
    d = to_dev(cuda, I, u0, U, S, GS)
    l1 = L().scan_backward_tiled(d[0], d[1], d[2], d[3], d[4], None, beta, 1.0, 0.0, 4.0, True, C=C)
    l2 = L().scan_backward_tiled(d[0], d[1], d[2], None, d[4], None, beta, 1.0, 0.0, 4.0, True, C=C)
    assert rel(_np(l1), ref) < TOL
    assert rel(_np(l2), ref) < TOL


def test_calls_from_a_fresh_thread(cuda):
    """A host thread whose first CUDA work is a library call (autograd's
    backward worker, when the caching allocator serves every allocation):
    the TMA descriptors must still encode, forward and backward."""
    import threading
    T, N = 4096, 1024
    I, u0, GS = gen(T, N, 0.05, 0.2, seed=17, grad=True)
    U, S = O.serial_forward(I, 0.99, 1.0, 0.0, u0)
    ref = O.serial_backward(I, u0, U, S, GS, None, 0.99, 1.0, 0.0, 4.0, True)
    d = to_dev(cuda, I, u0, U, GS)
    # warm the caching allocator with blocks of the sizes the calls allocate
    for _ in range(2):
        L().serial_forward(d[0], 0.99, 1.0, 0.0, d[1])
        L().scan_backward_tiled(d[0], d[1], d[2], None, d[3], None, 0.99, 1.0, 0.0, 4.0, True, C=1024)
    torch.cuda.synchronize()
    out = {}

    def body():
        try:
            out["fwd"] = L().serial_forward(d[0], 0.99, 1.0, 0.0, d[1])
            out["bwd"] = L().scan_backward_tiled(d[0], d[1], d[2], None, d[3], None, 0.99, 1.0, 0.0, 4.0, True,
                                                 C=1024)
        except Exception as e:  # noqa: BLE001 - reported below
            out["err"] = e

    th = threading.Thread(target=body)
    th.start()
    th.join()
    assert "err" not in out, out.get("err")
    torch.cuda.synchronize()
    assert_bit_equal(_np(out["fwd"][0]), U, "U")
    assert rel(_np(out["bwd"]), ref) < TOL


@pytest.mark.parametrize("N,T,C", ((16384, 1024, 1024), (1000, 4096, 512), (777, 2048, 2048), (777, 2048, 256),
                                   (64, 1 << 15, 4096)))
def test_v_path(cuda, N, T, C):
    """lif_tuned's V-saving path: V is the forward's pre-reset potential bit
    for bit, S unchanged, and the adjoint from V and GS alone (one sweep or
    chunks + fix-up; N = 777 takes the plain-kernel fallback) matches the
    oracle's serial adjoint."""
    beta = 0.99
    I, u0, GS = gen(T, N, 0.05, 0.2, seed=23, u0_sd=0.3, grad=True)
    Us, Ss, Vs = O.serial_forward(I, beta, 1.0, 0.0, u0, want_v=True)
    ref = O.serial_backward(I, u0, Us, Ss, GS, None, beta, 1.0, 0.0, 4.0, True)
    Id, u0d, GSd = to_dev(cuda, I, u0, GS)
    V, S = L().serial_forward_v(Id, beta, 1.0, 0.0, u0d)
    assert_bit_equal(_np(V), Vs, "V")
    assert_bit_equal(_np(S), Ss, "S")
    lam = L().lif_backward_v(V, GSd, beta, 1.0, 4.0, C=C)
    assert rel(_np(lam), ref) < TOL


@pytest.mark.parametrize("mode", ("scan", "serial"))
def test_lif_tuned_v_path_selected(cuda, mode):
    """At config 2's shape lif_tuned's forward is the single pass and saves V."""
    T, N = 1024, 16384
    I, u0, GS = gen(T, N, 0.05, 0.2, seed=4, grad=True)
    Us, Ss = O.serial_forward(I, 0.99, 1.0, 0.0, u0)
    dI_ref = O.serial_backward(I, u0, Us, Ss, GS, None, 0.99, 1.0, 0.0, 4.0, True)
    Id, u0d, GSd = to_dev(cuda, I, u0, GS)
    Id.requires_grad_(True)
    S = L().lif_tuned(Id, u0d, beta=0.99, mode=mode)
    assert S.grad_fn is not None and len(S.grad_fn.saved_tensors) == 1  # V only
    torch.autograd.backward(S, GSd)
    assert_bit_equal(_np(S), Ss, "S")
    assert rel(_np(Id.grad), dI_ref) < TOL


@pytest.mark.parametrize("beta,mu,sd", ((0.99, 0.05, 0.2), (1.0, -0.01, 0.05), (0.5, 0.4, 0.2)))
@pytest.mark.parametrize("N,T", ((4096, 1024), (1024, 1000), (2048, 4096), (512, 64), (1024, 200)))
def test_v_path_one_chunk_regimes(cuda, beta, mu, sd, N, T):
    """One-chunk adjoint from V across regimes: ragged tiles (T = 1000, 200),
    long spike-free stretches (beta = 1, negative drift), frequent spikes, and
    short sequences."""
    I, u0, GS = gen(T, N, mu, sd, seed=29, u0_sd=0.3, grad=True)
    Us, Ss, Vs = O.serial_forward(I, beta, 1.0, 0.0, u0, want_v=True)
    ref = O.serial_backward(I, u0, Us, Ss, GS, None, beta, 1.0, 0.0, 4.0, True)
    Vd, GSd = to_dev(cuda, Vs, GS)
    lam = L().lif_backward_v(Vd, GSd, beta, 1.0, 4.0, C=T)
    assert rel(_np(lam), ref) < TOL
