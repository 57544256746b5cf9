"""mxgg: Blackwell-native (sm_100a) MXFP8 grouped-GEMM kernels for MoE layers.

The public drop-in surface mirrors indianspeedster/grouped-gemms:
``kernels.triton_mxfp8_grouped_mm``, ``kernels.triton_mxfp8_wgrad`` and
``utils.to_mx`` (the sibling ``kernels`` package and ``utils`` module).  This
package holds the implementation: the ctypes binding of ``libmxgg.so`` and the
torch custom ops built on it.
"""

from . import _lib, ops
from ._lib import MxggError, device_status, set_schedule, set_tile_config, set_wait_limit, wait_limit
from .ops import (build_tile_map, grouped_mm_mx_op, grouped_mm_op, grouped_mm_segments_op, to_mx_fp4_op,
                  to_mx_op, wgrad_accumulate_op, wgrad_op)


def available() -> bool:
    """True when libmxgg.so loads and the current CUDA device is sm_100."""
    import torch
    if not torch.cuda.is_available():
        return False
    try:
        _lib.load()
    except Exception:
        return False
    return torch.cuda.get_device_capability() == (10, 0)


__all__ = ["MxggError", "available", "build_tile_map", "device_status", "grouped_mm_mx_op", "grouped_mm_op",
           "grouped_mm_segments_op", "ops", "set_tile_config", "set_schedule", "set_wait_limit", "to_mx_fp4_op",
           "to_mx_op", "wait_limit", "wgrad_accumulate_op", "wgrad_op"]
