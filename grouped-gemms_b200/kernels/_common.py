"""Availability probe shared by the grouped-GEMM entry points.

Mirrors the reference's ``kernels/_common.py:17-27``.  The exported name
``_rocm_mxfp8_available`` is kept so callers written against the reference
keep importing; here it is True when the sm_100a library loads and the
current device is a B200-class GPU (compute capability 10.0).
"""

import mxgg

_UNAVAILABLE_MSG = "MXFP8 grouped-GEMM kernels require an sm_100 (B200) GPU and the built libmxgg.so"

_mxfp8_available = mxgg.available()
_rocm_mxfp8_available = _mxfp8_available


def _scale_layout(name: str) -> int:
    """``scale_layout`` keyword -> the library's constant."""
    from mxgg import _lib
    layouts = {"row_major": _lib.SCALE_ROW_MAJOR, "blocked": _lib.SCALE_BLOCKED}
    if name not in layouts:
        raise ValueError(f"scale_layout must be 'row_major' or 'blocked', got {name!r}")
    return layouts[name]
