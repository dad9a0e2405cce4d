"""The no-allocation scan forward (lifb_scan_fwd_v3_noalloc) against the
regular entry point (lifb_scan_fwd_v3 with a caller workspace).

The no-allocation variant exists for callers that cannot allocate device
memory at call time (a plain C/FFI host without a device allocator, a
process whose device memory is committed elsewhere, a loop that must never
call cudaMalloc).  Its scratch is a fixed array inside the library, so the
test checks two calls in a row, on different inputs, each bit-identical to
the regular entry point on the same inputs (the forward's outputs are exact,
so the tolerance is zero), and that oversized requests are refused.

This file is collected last on purpose: it must pass when run alone in a
fresh process and after every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _lib():
    from hard_resets_compose_b200 import _lib as lb
    return lb.load()


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _regular(L, I, u0, beta, C, K, max_repair=-1, stats=None):
    T, N = I.shape
    U = torch.empty_like(I)
    S = torch.empty_like(I)
    nb = L.lifb_scan_fwd_v3_workspace_bytes(T, N, C, K)
    ws = torch.empty(nb, dtype=torch.uint8, device=I.device)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.lifb_scan_fwd_v3(_p(I), _p(u0), _p(U), _p(S), T, N, beta, 1.0, 0.0, C, K, max_repair, _p(ws), nb,
                            _p(stats), st)
    assert rc == 0, L.lifb_last_error()
    return U, S


def _noalloc(L, I, u0, beta, C, K, max_repair=-1, stats=None):
    T, N = I.shape
    U = torch.empty_like(I)
    S = torch.empty_like(I)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = L.lifb_scan_fwd_v3_noalloc(_p(I), _p(u0), _p(U), _p(S), T, N, beta, 1.0, 0.0, C, K, max_repair,
                                    _p(stats), st)
    assert rc == 0, L.lifb_last_error()
    return U, S


def test_noalloc_matches_regular_entry_on_two_calls(cuda):
    L = _lib()
    # M = T/C = 16 chunks, so the scan uses its scratch (maps, starts, ends)
    cases = [(1024, 4096, 0.1, 0.3, 0.9, 0), (2048, 1000, 0.05, 0.2, 0.99, 1)]
    for (T, N, mu, sd, beta, seed) in cases:
        C, K = 64 if T == 1024 else 128, 16
        assert L.lifb_scan_fwd_v3_workspace_bytes(T, N, C, K) <= (64 << 20)
        I_np, u0_np = O.gen_inputs(T, N, mu, sd, seed=seed)
        I = torch.from_numpy(I_np).to(cuda)
        u0 = torch.from_numpy(u0_np).to(cuda)
        Ur, Sr = _regular(L, I, u0, beta, C, K)
        Un, Sn = _noalloc(L, I, u0, beta, C, K)
        torch.cuda.synchronize()
        assert torch.equal(Un.view(torch.int32), Ur.view(torch.int32))
        assert torch.equal(Sn.view(torch.int32), Sr.view(torch.int32))
    # and both equal the serial recurrence (the last case's inputs)
    Us, Ss = O.serial_forward(I_np, beta, 1.0, 0.0, u0_np)
    assert np.array_equal(Un.cpu().numpy().view(np.uint32), Us.view(np.uint32))
    assert np.array_equal(Sn.cpu().numpy().view(np.uint32), Ss.view(np.uint32))


def test_noalloc_stats_and_capped_repair_paths(cuda):
    """The paths that read chunk starts and ends across repair rounds: a stats
    buffer (device counters) and max_repair >= 0 (rounds capped as the
    reference's `repair`).  Each runs right after a call on other inputs has
    left different values in the shared scratch, and must equal the regular
    entry point bit for bit, outputs and stats alike."""
    from hard_resets_compose_b200 import _lib as lb
    L = _lib()
    T, N, C, K = 4096, 512, 64, 16
    for seed, (mu, sd, beta), max_repair in ((3, (0.15, 0.4, 0.9), 10 ** 6), (4, (-0.1, 0.6, 0.99), 2),
                                              (5, (0.4, 0.2, 0.5), 0)):
        I_np, u0_np = O.gen_inputs(T, N, mu, sd, seed=seed, u0_sd=0.3)
        I = torch.from_numpy(I_np).to(cuda)
        u0 = torch.from_numpy(u0_np).to(cuda)
        # leave other values in the scratch first
        J = torch.from_numpy(O.gen_inputs(T, N, 0.3, 0.5, seed=seed + 100)[0]).to(cuda)
        _noalloc(L, J, u0, 0.95, C, K, max_repair=max_repair, stats=torch.zeros(lb.STATS_BYTES, dtype=torch.uint8,
                                                                               device=cuda))
        sr = torch.zeros(lb.STATS_BYTES, dtype=torch.uint8, device=cuda)
        sn = torch.zeros(lb.STATS_BYTES, dtype=torch.uint8, device=cuda)
        Ur, Sr = _regular(L, I, u0, beta, C, K, max_repair=max_repair, stats=sr)
        Un, Sn = _noalloc(L, I, u0, beta, C, K, max_repair=max_repair, stats=sn)
        torch.cuda.synchronize()
        assert torch.equal(Un.view(torch.int32), Ur.view(torch.int32))
        assert torch.equal(Sn.view(torch.int32), Sr.view(torch.int32))
        assert torch.equal(sn, sr), "device stats differ"
        st = lb.read_stats(sn)
        assert st.n_maps > 0


def test_noalloc_allocates_nothing(cuda):
    """Free device memory is the same before and after a call that uses the
    scratch (stats force the map pipeline, which carves it)."""
    from hard_resets_compose_b200 import _lib as lb
    L = _lib()
    T, N, C, K = 2048, 1000, 128, 16
    I_np, u0_np = O.gen_inputs(T, N, 0.05, 0.2, seed=7)
    I = torch.from_numpy(I_np).to(cuda)
    u0 = torch.from_numpy(u0_np).to(cuda)
    U = torch.empty_like(I)
    S = torch.empty_like(I)
    stats = torch.zeros(lb.STATS_BYTES, dtype=torch.uint8, device=cuda)
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    args = (_p(I), _p(u0), _p(U), _p(S), T, N, 0.99, 1.0, 0.0, C, K, -1, _p(stats), st)
    assert L.lifb_scan_fwd_v3_noalloc(*args) == 0  # warm-up: first-call set-up, kernel modules
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(cuda)
    assert L.lifb_scan_fwd_v3_noalloc(*args) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(cuda)
    assert free1 == free0


def test_noalloc_rejects_requests_above_its_scratch(cuda):
    L = _lib()
    T, N, C, K = 1024, 1 << 20, 64, 16  # ~2.6 GB of scratch
    assert L.lifb_scan_fwd_v3_workspace_bytes(T, N, C, K) > (64 << 20)
    fake = ctypes.c_void_p(256)  # never dereferenced: the size check comes first
    rc = L.lifb_scan_fwd_v3_noalloc(fake, fake, fake, fake, T, N, 0.9, 1.0, 0.0, C, K, -1, None, None)
    assert rc == 1
    assert b"no-allocation scratch" in L.lifb_last_error()
