"""The C-ABI library loads and exports every symbol include/*.h declares
(no GPU needed: only host-side paths are called here)."""
import ctypes
import glob
import os
import re

import pytest

from hard_resets_compose_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    syms = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"\b(lifb_\w+)\s*\(", text):
            syms.add(m.group(1))
    return sorted(syms)


def test_header_declares_entry_points():
    syms = declared_symbols()
    for s in ("lifb_serial_fwd", "lifb_serial_bwd", "lifb_scan_fwd_v3", "lifb_scan_fwd_v4", "lifb_scan_bwd"):
        assert s in syms


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    missing = [s for s in declared_symbols() if not hasattr(L, s)]
    assert not missing, f"liblifb.so lacks {missing}"
    # and the ctypes table covers every declared entry point
    assert set(declared_symbols()) <= set(_lib.SIGNATURES)


def test_abi_version_and_status_strings():
    L = _lib.load()
    assert L.lifb_abi_version() == _lib.ABI_VERSION
    for code in range(6):
        assert L.lifb_status_string(code)
    assert L.lifb_status_string(99) == b"unknown status"


def test_workspace_sizes():
    L = _lib.load()
    T, N, C, K = 1024, 4096, 64, 16
    M = T // C
    nb = L.lifb_scan_fwd_v3_workspace_bytes(T, N, C, K)
    assert nb >= (2 * K + 7) * M * N * 4
    assert L.lifb_scan_fwd_v3_workspace_bytes(T, N, 48, K) == 0  # T % C != 0
    assert L.lifb_scan_fwd_v4_workspace_bytes(8192, 777, 64, 16, 16, 32) > 0
    assert L.lifb_scan_fwd_v4_workspace_bytes(8192, 777, 64, 3, 16, 32) == 0
    assert L.lifb_scan_bwd_workspace_bytes(T, N, 64) >= 3 * M * N * 4


def test_argument_errors_return_status_without_touching_a_gpu():
    L = _lib.load()
    null = None
    # negative shape
    st = L.lifb_serial_fwd(null, null, null, null, -1, 4, 0.9, 1.0, 0.0, null)
    assert st == 1 and b"negative" in L.lifb_last_error()
    # T not a multiple of C (checked before any CUDA call)
    fake = ctypes.c_void_p(256)
    st = L.lifb_scan_fwd_v3(fake, fake, fake, fake, 100, 8, 0.9, 1.0, 0.0, 64, 16, -1, null, 0, null, null)
    assert st == 1 and b"multiple" in L.lifb_last_error()
    # capacity out of range
    st = L.lifb_scan_fwd_v3(fake, fake, fake, fake, 128, 8, 0.9, 1.0, 0.0, 64, 65, -1, null, 0, null, null)
    assert st == 1
    # v4 group mismatch
    st = L.lifb_scan_fwd_v4(fake, fake, fake, fake, 128, 8, 0.9, 1.0, 0.0, 64, 3, 16, 32, -1, null, 0, null, null)
    assert st == 1
    # empty problems are a no-op success
    assert L.lifb_serial_fwd(null, null, null, null, 0, 16, 0.9, 1.0, 0.0, null) == 0
    assert L.lifb_scan_bwd(null, null, null, null, null, null, null, 0, 16, 0.9, 1.0, 0.0, 4.0, 1, 64, null, 0,
                           null) == 0


def test_python_api_refuses_cpu_tensors():
    import torch
    from hard_resets_compose_b200 import lifscan as L
    I = torch.zeros(64, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        L.serial_forward(I, 0.9, 1.0, 0.0, torch.zeros(4))
    with pytest.raises(RuntimeError, match="CUDA"):
        L.lif_tuned(I, torch.zeros(4))
