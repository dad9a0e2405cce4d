"""The host-side policies of hard_resets_compose_b200.lifscan, on the CPU:
_pick_C (the reference's rule, lifscan/triton_lif.py:647-651), auto_modes
(the reference's rule with B200 thresholds, :997-1000), and the B200 chunk
and segment policies that scan_forward_auto, scan_backward_auto and lif_tuned
use. Every choice must be admissible for the kernels it feeds: chunks divide
T, segments are long enough for their lead-ins, and the boundaries fall where
the constants say."""
import pytest

from hard_resets_compose_b200 import lifscan as L


def _pick_c_rule(T, D):
    """_pick_C restated: the largest C in (256, 128, ..., 8) with T % C == 0,
    C % D == 0 and C*C <= 4T."""
    for C in (256, 128, 64, 32, 16, 8):
        if T % C == 0 and C % D == 0 and C * C <= 4 * T:
            return C
    return None


@pytest.mark.parametrize("T", (8, 16, 64, 100, 256, 1000, 1024, 4096, 65536, 1 << 20, 3 * 512))
@pytest.mark.parametrize("D", (1, 2, 8, 16))
def test_pick_c_follows_the_reference_rule(T, D):
    want = _pick_c_rule(T, D)
    if want is None:
        with pytest.raises(ValueError):
            L._pick_C(T, D)
    else:
        assert L._pick_C(T, D) == want


def test_auto_modes_thresholds():
    N, T = L.AUTO_FWD_MAX_N, L.AUTO_FWD_MIN_T
    assert L.auto_modes(N, T)[0] == "scan"
    assert L.auto_modes(N + 1, T)[0] == "serial"
    assert L.auto_modes(N, T - 1)[0] == "serial"
    N, T = L.AUTO_BWD_MAX_N, L.AUTO_BWD_MIN_T
    assert L.auto_modes(N, T)[1] == "scan"
    assert L.auto_modes(N + 1, T)[1] == "serial"
    assert L.auto_modes(N, T - 1)[1] == "serial"


@pytest.mark.parametrize("N", (1, 100, 1024, 8191, 8192, 16384, 1 << 20))
@pytest.mark.parametrize("T", (7, 64, 1000, 1024, 4096, 1 << 17, 1 << 20))
def test_backward_chunk_divides_t(N, T):
    C = L.scan_chunk_bwd(T, N)
    assert 1 <= C <= T and T % C == 0
    if N >= L.SCAN_BWD_SERIAL_MIN_N:
        assert C == T  # one chunk: the streaming pass fills the GPU
    elif C < T:
        # halved only while fewer (chunk, 32-neuron) warps than wanted were in flight
        assert (T // C) // 2 < max(1, -(-8 * 148 * 32 // N))


@pytest.mark.parametrize("N", (1, 1024, 16384, 37887, 37888, 1 << 20))
@pytest.mark.parametrize("T", (1024, 4096, 8192, 16384, 1 << 17, 1 << 20, 3 * 4096))
def test_speculative_segments(N, T):
    Lseg, W = L.spec_segment(T, N)
    if Lseg == T:
        assert W == 0  # the single streaming pass
        if N < L.SPEC_FILL and T % L.SPEC_MIN_L == 0:
            assert T // L.SPEC_MIN_L < 2  # no admissible segment length
    else:
        assert N < L.SPEC_FILL
        assert T % Lseg == 0 and T // Lseg >= 2
        assert L.SPEC_MIN_L <= Lseg <= L.SPEC_L and Lseg & (Lseg - 1) == 0
        assert W == min(L.SPEC_LEAD, Lseg)


def test_wide_problems_take_the_single_pass():
    assert L.spec_segment(1 << 20, L.SPEC_FILL) == (1 << 20, 0)
    assert L.scan_chunk_fwd(1024, 16384) == 1024


def test_block_leadin_policy():
    """The block-level lead-in forward is chosen for short sequences with few
    neurons when its lead-in (grown like 1/(-ln beta)) keeps the chain under
    half of T; otherwise the single pass or the long-sequence path."""
    from hard_resets_compose_b200 import lifscan as L
    assert L.block_leadin(1024, 4096, 0.9) == (64, 256)   # config 1
    assert L.block_leadin(1024, 4096, 0.5) == (64, 64)
    assert L.block_leadin(1024, 4096, 0.99) == (0, 0)     # lead-in longer than half of T
    assert L.block_leadin(1024, 16384, 0.9) == (0, 0)     # the single pass fills the GPU
    assert L.block_leadin(1024, 4097, 0.9) == (0, 0)      # no TMA path (N % 4)
    assert L.block_leadin(4096, 4096, 0.9) == (0, 0)      # the slab no longer fits on chip
    assert L.block_leadin(1024, 4096, 1.0) == (0, 0)
