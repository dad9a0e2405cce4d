"""ctypes binding of liblifb.so (include/lifscan_b200.h).

The product path calls CUDA only through this C ABI.  There is no CPU or
Python fallback: if the library is missing or a tensor is not on a CUDA
device, the call raises.
"""
from __future__ import annotations

import ctypes
import os
import threading

import torch

from . import build as _build

_lock = threading.Lock()
_lib = None

c_void_p = ctypes.c_void_p
c_i64 = ctypes.c_int64
c_int = ctypes.c_int
c_float = ctypes.c_float
c_size_t = ctypes.c_size_t

ABI_VERSION = 1

# Every symbol include/lifscan_b200.h declares, with its ctypes signature.
SIGNATURES = {
    "lifb_abi_version": ([], c_int),
    "lifb_kernel_launches": ([], ctypes.c_uint64),
    "lifb_status_string": ([c_int], ctypes.c_char_p),
    "lifb_last_error": ([], ctypes.c_char_p),
    "lifb_device_status": ([c_int], c_int),
    "lifb_check_device": ([c_int], c_int),
    "lifb_poll_device": ([], c_int),
    "lifb_serial_fwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float,
                         c_void_p], c_int),
    "lifb_serial_bwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64,
                         c_float, c_float, c_float, c_float, c_int, c_void_p], c_int),
    "lifb_scan_fwd_v3_workspace_bytes": ([c_i64, c_i64, c_int, c_int], c_size_t),
    "lifb_scan_fwd_v3": ([c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float,
                          c_int, c_int, c_int, c_void_p, c_size_t, c_void_p, c_void_p], c_int),
    "lifb_scan_fwd_v4_workspace_bytes": ([c_i64, c_i64, c_int, c_int, c_int, c_int], c_size_t),
    "lifb_scan_fwd_v4": ([c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float,
                          c_int, c_int, c_int, c_int, c_int, c_void_p, c_size_t, c_void_p, c_void_p], c_int),
    "lifb_scan_fwd_v3_noalloc": ([c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float,
                                  c_float, c_int, c_int, c_int, c_void_p, c_void_p], c_int),
    "lifb_lif_fwd_bwd_host_workspace_bytes": ([c_i64, c_i64, c_i64], c_size_t),
    "lifb_lif_fwd_bwd_host": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float,
                               c_float, c_float, c_float, c_i64, c_void_p, c_size_t, c_void_p], c_int),
    "lifb_dense_dgrad_workspace_bytes": ([c_i64, c_i64], c_size_t),
    "lifb_dense_dgrad": ([c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_void_p, c_size_t, c_void_p], c_int),
    "lifb_lif_fwd_bwd_host_rows_block": ([c_i64, c_i64], c_i64),
    "lifb_lif_fwd_bwd_host_rows_workspace_bytes": ([c_i64, c_i64, c_i64], c_size_t),
    "lifb_lif_fwd_bwd_host_rows": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64,
                                    c_float, c_float, c_float, c_float, c_i64, c_void_p, c_size_t, c_void_p], c_int),
    "lifb_scan_bwd_workspace_bytes": ([c_i64, c_i64, c_int], c_size_t),
    "lifb_scan_bwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64,
                       c_float, c_float, c_float, c_float, c_int, c_int, c_void_p, c_size_t, c_void_p], c_int),
    "lifb_scan_fwd_spec_workspace_bytes": ([c_i64, c_i64, c_i64], c_size_t),
    "lifb_scan_fwd_spec": ([c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float, c_i64,
                            c_i64, c_void_p, c_i64, c_void_p, c_size_t, c_void_p], c_int),
    "lifb_scan_fwd_spec_begin": ([c_void_p, c_i64, c_i64, c_float, c_float, c_float, c_i64, c_i64, c_void_p,
                                  c_void_p, c_size_t, c_void_p], c_int),
    "lifb_scan_fwd_spec_finish": ([c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float,
                                   c_i64, c_void_p, c_size_t, c_void_p], c_int),
    "lifb_param_grad_chunks": ([c_i64, c_i64], c_int),
    "lifb_param_grad_partials": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float,
                                  c_float, c_float, c_int, c_void_p], c_int),
    "lifb_serial_fwd_v": ([c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float,
                           c_void_p], c_int),
    "lifb_lif_bwd_v_workspace_bytes": ([c_i64, c_i64, c_int], c_size_t),
    "lifb_lif_bwd_v": ([c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float, c_int, c_void_p,
                        c_size_t, c_void_p], c_int),
    "lifb_soft_serial_fwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_void_p],
                             c_int),
    "lifb_soft_scan_fwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_i64, c_i64,
                           c_void_p, c_size_t, c_void_p], c_int),
    "lifb_soft_serial_bwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float,
                             c_float, c_void_p], c_int),
    "lifb_soft_adjoint_v": ([c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float, c_void_p], c_int),
    "lifb_aff_serial_fwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float,
                             c_float, c_void_p], c_int),
    "lifb_aff_scan_fwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float, c_float,
                           c_i64, c_i64, c_void_p, c_size_t, c_void_p], c_int),
    "lifb_aff_adjoint": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float,
                          c_float, c_void_p], c_int),
    "lifb_aff_param_grad_partials": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64,
                                      c_float, c_float, c_float, c_int, c_void_p], c_int),
    "lifb_reverse_linear_scan": ([c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_void_p], c_int),
    "lifb_aff_serial_fwd_v": ([c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float,
                               c_float, c_void_p], c_int),
    "lifb_aff_adjoint_v": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float,
                            c_float, c_float, c_float, c_void_p], c_int),
    "lifb_alif_serial_fwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float,
                              c_float, c_float, c_float, c_float, c_void_p], c_int),
    "lifb_alif_scan_fwd_workspace_bytes": ([c_i64, c_i64, c_i64], c_size_t),
    "lifb_alif_scan_fwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float,
                            c_float, c_float, c_float, c_float, c_i64, c_i64, c_void_p, c_i64, c_void_p, c_size_t,
                            c_void_p], c_int),
    "lifb_alif_warm_predict": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64,
                                c_i64, c_float, c_float, c_float, c_float, c_float, c_float, c_float, c_void_p],
                               c_int),
    "lifb_alif_bwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                       c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float, c_float, c_float, c_void_p],
                      c_int),
    "lifb_alif_bwd_scan_workspace_bytes": ([c_i64, c_i64, c_i64], c_size_t),
    "lifb_alif_bwd_scan": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                            c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float, c_float, c_float,
                            c_i64, c_void_p, c_size_t, c_void_p], c_int),
    "lifb_leaky_fwd": ([c_void_p, c_void_p, c_i64, c_i64, c_float, c_void_p], c_int),
    "lifb_leaky_bwd": ([c_void_p, c_void_p, c_i64, c_i64, c_float, c_void_p], c_int),
    "lifb_spike_mask_stride": ([c_i64], c_i64),
    "lifb_spike_mask": ([c_void_p, c_void_p, c_i64, c_i64, c_void_p], c_int),
    "lifb_spike_linear_lif_fwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                   c_i64, c_i64, c_i64, c_i64, c_float, c_float, c_float, c_void_p], c_int),
    "lifb_spike_linear_wgrad_workspace_bytes": ([c_i64, c_i64, c_i64], c_size_t),
    "lifb_spike_linear_wgrad": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_i64, c_void_p,
                                 c_size_t, c_void_p], c_int),
    "lifb_tshard_fwd_tail": ([c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float, c_float, c_i64, c_i64,
                              c_void_p, c_void_p, c_size_t, c_void_p], c_int),
    "lifb_tshard_fwd_head": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float,
                              c_float, c_i64, c_void_p, c_size_t, c_void_p], c_int),
    "lifb_tshard_workspace_bytes": ([c_i64, c_i64, c_int, c_int, c_int, c_int], c_size_t),
    "lifb_tshard_envelope": ([c_void_p, c_i64, c_i64, c_int, c_int, c_int, c_int, c_float, c_float, c_void_p,
                              c_void_p, c_size_t, c_void_p], c_int),
    "lifb_tshard_slice_map": ([c_void_p, c_void_p, c_int, c_void_p, c_i64, c_i64, c_float, c_float, c_float, c_int,
                               c_int, c_int, c_int, c_int, c_void_p, c_void_p, c_size_t, c_void_p], c_int),
    "lifb_tshard_apply": ([c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                           c_i64, c_i64, c_float, c_float, c_float, c_int, c_int, c_int, c_int, c_void_p, c_size_t,
                           c_void_p], c_int),
    "lifb_tshard_repair": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float,
                            c_float, c_float, c_void_p], c_int),
    "lifb_tshard_bwd_workspace_bytes": ([c_i64, c_i64, c_int], c_size_t),
    "lifb_tshard_bwd": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float, c_float,
                         c_float, c_float, c_int, c_void_p, c_size_t, c_void_p], c_int),
    "lifb_tshard_bwd_fix": ([c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_i64, c_i64, c_float,
                             c_float, c_float, c_int, c_void_p, c_size_t, c_void_p], c_int),
}


LIFB_ERR_DEVICE = 5


class LifbError(RuntimeError):
    """A nonzero status returned by liblifb.  `status` is the library's
    status code; for a device-side error (LIFB_ERR_DEVICE) `device_code` is
    the code a kernel recorded (101: a bounded wait for an asynchronous copy
    expired), else None."""

    def __init__(self, msg, status=None, device_code=None):
        super().__init__(msg)
        self.status = status
        self.device_code = device_code


def lib_path() -> str:
    return _build.LIB


def bind(path: str):
    """ctypes handle of a liblifb build at `path` with every declared
    signature set (the product library, or a test build of it)."""
    L = ctypes.CDLL(path)
    for name, (args, res) in SIGNATURES.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    v = L.lifb_abi_version()
    if v != ABI_VERSION:
        raise RuntimeError(f"liblifb ABI version {v} != expected {ABI_VERSION}")
    return L


def load(build_if_missing: bool = True):
    """Load liblifb.so (building it first when it is missing or stale and nvcc
    is available).  Raises if it cannot be loaded."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB
        if build_if_missing:
            try:
                path = _build.build()
            except (RuntimeError, OSError) as e:  # no nvcc: use the prebuilt library if present
                if not os.path.exists(path):
                    raise RuntimeError(f"liblifb.so is missing and cannot be built: {e}") from e
        if not os.path.exists(path):
            raise RuntimeError(f"liblifb.so not found at {path}; run python -m hard_resets_compose_b200.build")
        _lib = bind(path)
        return _lib


def check(status: int, what: str, lib=None) -> None:
    if status != 0:
        L = lib or load(False)
        msg = L.lifb_last_error().decode() or L.lifb_status_string(status).decode()
        code = None
        if status == LIFB_ERR_DEVICE:
            import re
            m = re.search(r"device status (-?\d+)", msg)
            code = int(m.group(1)) if m else None
        raise LifbError(f"{what} failed (status {status}: {L.lifb_status_string(status).decode()}): {msg}",
                        status=status, device_code=code)


def check_device(what: str, reset: bool = False, lib=None) -> None:
    """Raises LifbError (status LIFB_ERR_DEVICE, device_code = the kernel's
    code) when a kernel of the library has reported a device-side error on
    the current device.  Synchronous: call it where the host waits anyway."""
    L = lib or load(False)
    check(L.lifb_check_device(int(bool(reset))), what, L)


def poll_device(what: str, lib=None) -> None:
    """The non-blocking form of check_device: raises for a device-side error
    seen by an earlier poll's asynchronous read, and starts the next read.
    Does nothing while the current stream is being captured into a graph."""
    if torch.cuda.is_current_stream_capturing():
        return
    L = lib or load(False)
    check(L.lifb_poll_device(), what, L)


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor):
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


class Stats(ctypes.Structure):
    """Mirror of lifb_stats."""
    _fields_ = [
        ("repair_iters", ctypes.c_int32),
        ("max_cnt", ctypes.c_int32),
        ("max_super_cnt", ctypes.c_int32),
        ("status", ctypes.c_int32),
        ("n_maps", ctypes.c_int64),
        ("n_overflow", ctypes.c_int64),
        ("sum_cnt", ctypes.c_int64),
        ("n_super", ctypes.c_int64),
        ("n_super_overflow", ctypes.c_int64),
        ("sum_super_cnt", ctypes.c_int64),
    ]


STATS_BYTES = ctypes.sizeof(Stats)


def read_stats(dev_buf: torch.Tensor) -> Stats:
    host = dev_buf.cpu()  # synchronises the stream
    return Stats.from_buffer_copy(bytes(host.numpy().tobytes()))
