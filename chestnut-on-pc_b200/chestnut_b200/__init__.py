"""chestnut_b200: B200-native frame engine for chestnut-class driving models.

The compute path is libchestnut.so (hand-written sm_100a CUDA: tcgen05 GEMMs,
HBM-streaming reductions, zero-border gathers, one CUDA graph per frame),
reached through ctypes.  See include/chestnut.h for the C ABI.
"""
from ._lib import ChestnutError, DeviceBuffer, PinnedArray, lib  # noqa: F401
from .engine import Engine, output_slices, param_table  # noqa: F401
