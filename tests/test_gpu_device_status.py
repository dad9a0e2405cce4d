"""Device-side wait timeouts reach the caller as an error.

Every kernel wait on an asynchronous copy is bounded; on expiry the kernel
records code 101 in the library's per-device status word and returns.  This
test builds a second copy of the library with a short wait limit and a
test-only entry point whose kernel waits on an mbarrier phase that nothing
completes (no copy is ever issued, so none is left in flight), then checks
that the check and poll entry points, and the Python layer above them, raise
LifbError with device code 101, and that the GPU context stays usable.  The
product library is not modified: the test build lives in a temporary
directory and has its own status word."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.helpers import assert_bit_equal, gen, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def test_lib(tmp_path_factory):
    from hard_resets_compose_b200 import _lib, build
    out = str(tmp_path_factory.mktemp("lifb_hooks") / "liblifb_hooks.so")
    # ~10 ms of SM clock instead of ~1 s
    build.build(out=out, defines=("LIFB_WAIT_CYCLES=20000000LL", "LIFB_TEST_HOOKS"))
    L = _lib.bind(out)
    L.lifb_test_stalled_wait.argtypes = [ctypes.c_void_p]
    L.lifb_test_stalled_wait.restype = ctypes.c_int
    return L


def test_expired_wait_raises_code_101(cuda, test_lib):
    from hard_resets_compose_b200 import _lib
    L = test_lib
    st = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    assert L.lifb_check_device(1) == 0  # clean start
    assert L.lifb_poll_device() == 0
    assert L.lifb_test_stalled_wait(st) == 0  # the launch itself succeeds
    torch.cuda.synchronize(cuda)
    # the non-blocking poll reports it once a read issued after the kernel has landed
    L.lifb_poll_device()
    torch.cuda.synchronize(cuda)
    L_poll = None
    for _ in range(1000):
        L_poll = L.lifb_poll_device()
        if L_poll:
            break
    assert L_poll == _lib.LIFB_ERR_DEVICE
    assert b"101" in L.lifb_last_error()
    with pytest.raises(_lib.LifbError) as ei:
        _lib.poll_device("after the stalled wait", lib=L)
    assert ei.value.status == _lib.LIFB_ERR_DEVICE and ei.value.device_code == 101
    # the synchronous check reports it too, and clears it on request
    with pytest.raises(_lib.LifbError) as ei:
        _lib.check_device("after the stalled wait", reset=True, lib=L)
    assert ei.value.device_code == 101
    assert L.lifb_check_device(0) == 0
    assert L.lifb_device_status(0) == 0


def test_context_usable_after_the_timeout(cuda, test_lib):
    """After the expired wait the same process still computes exact results,
    through the test build and through the product library."""
    from hard_resets_compose_b200 import _lib
    L = test_lib
    st = ctypes.c_void_p(torch.cuda.current_stream(cuda).cuda_stream)
    assert L.lifb_test_stalled_wait(st) == 0
    torch.cuda.synchronize(cuda)
    assert L.lifb_check_device(1) == _lib.LIFB_ERR_DEVICE
    T, N = 1024, 512
    I, u0 = gen(T, N, 0.1, 0.3, seed=2)
    Us, Ss = O.serial_forward(I, 0.9, 1.0, 0.0, u0)
    Id, u0d = to_dev(cuda, I, u0)
    for lib in (L, _lib.load()):
        U = torch.empty_like(Id)
        S = torch.empty_like(Id)
        assert lib.lifb_serial_fwd(_lib.ptr(Id), _lib.ptr(u0d), _lib.ptr(U), _lib.ptr(S), T, N, 0.9, 1.0, 0.0, st) == 0
        torch.cuda.synchronize(cuda)
        assert lib.lifb_check_device(0) == 0
        assert_bit_equal(U.cpu().numpy(), Us, "U")
        assert_bit_equal(S.cpu().numpy(), Ss, "S")


def test_product_paths_check_the_device(cuda):
    """The Python layer reads the status where it synchronises anyway (stats
    read-back, lif_tuned_host) and polls it after every autograd backward:
    on a healthy run these pass silently."""
    from hard_resets_compose_b200 import _lib, lifscan as Lm
    assert _lib.load().lifb_check_device(1) == 0
    I, u0, GS = gen(256, 64, 0.1, 0.3, seed=3, grad=True)
    Id, u0d, GSd = to_dev(cuda, I, u0, GS)
    st = {}
    Lm.scan_forward_v3(Id, 0.9, 1.0, 0.0, u0d, C=64, K=16, stats=st)
    Iq = Id.clone().requires_grad_(True)
    S = Lm.lif_tuned(Iq, u0d, beta=0.9)
    torch.autograd.backward(S, GSd)
    torch.cuda.synchronize(cuda)
    Sh, dIh, du0h = Lm.lif_tuned_host(torch.from_numpy(I), torch.from_numpy(GS), beta=0.9)
    assert np.array_equal(Sh.numpy(), S.detach().cpu().numpy())
