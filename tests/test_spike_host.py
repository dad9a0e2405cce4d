"""Host logic of the spike-input layers (hard_resets_compose_b200/shdnet.py),
without a GPU: when a layer's carried spike mask is trusted, when the fused
producer applies, and the mask-format stride of the C ABI."""
import torch

from hard_resets_compose_b200 import shdnet


def test_carried_mask_follows_the_tensor_version():
    x = torch.zeros(4, 3, 8)
    assert shdnet._carried_mask(x) is None
    m = torch.zeros(12, 4, dtype=torch.int32)
    setattr(x, shdnet._MASK_ATTR, (m, x._version))
    assert shdnet._carried_mask(x) is m
    x.add_(1.0)  # an in-place change: the mask no longer describes x
    assert shdnet._carried_mask(x) is None
    y = x.view(12, 8)  # another tensor object carries no mask
    assert shdnet._carried_mask(y) is None


def test_spike_producer_applies():
    assert shdnet.spike_producer_applies(700, 256)
    assert shdnet.spike_producer_applies(256, 256)
    assert shdnet.spike_producer_applies(1024, 32)
    assert not shdnet.spike_producer_applies(1025, 256)  # the weight slice must fit in shared memory
    assert not shdnet.spike_producer_applies(700, 20)  # 32 outputs per warp
    assert not shdnet.spike_producer_applies(0, 256)


def test_mask_stride_is_whole_16_byte_units():
    from hard_resets_compose_b200 import _lib
    lib = _lib.load(build_if_missing=False)
    for d, want in ((1, 4), (31, 4), (32, 4), (96, 4), (97, 8), (700, 24), (256, 12), (1024, 36)):
        s = lib.lifb_spike_mask_stride(d)
        assert s == want, (d, s)
        assert s % 4 == 0 and s >= (d + 31) // 32 + 1
    assert lib.lifb_spike_mask_stride(0) == 0
