"""B200-native (sm_100a) exact map-space scan for hard-reset LIF neurons.

Public API: ``hard_resets_compose_b200.lifscan`` mirrors the reference's
``lifscan.triton_lif`` (scan_forward_v3/v4, scan_backward_tiled, lif_tuned,
serial_* and lif_auto); ``hard_resets_compose_b200.shdnet`` holds the
700-256-256-20 network that consumes it.  All compute runs in liblifb.so
(C ABI in include/lifscan_b200.h).
"""
__version__ = "0.1.0"
