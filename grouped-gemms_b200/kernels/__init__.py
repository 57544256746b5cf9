"""Blackwell MXFP8 grouped-GEMM kernels (drop-in for the reference's ``kernels`` package).

Public entry points (reference ``kernels/__init__.py:17-25``):
  - ``triton_mxfp8_grouped_mm``: forward + dgrad grouped GEMM (A @ B^T per group)
  - ``triton_mxfp8_wgrad``: weight-gradient grouped GEMM (A^T @ B per group)
  - ``mxfp8_grouped_mm_to_mx``: the forward with ``to_mx`` of its output fused
    into the epilogue (no reference counterpart)
  - ``_rocm_mxfp8_available``: kept name; True when the sm_100a kernels can run.
"""

from ._common import _mxfp8_available, _rocm_mxfp8_available
from .backward import triton_mxfp8_wgrad
from .forward import mxfp8_grouped_mm_to_mx, triton_mxfp8_grouped_mm

__all__ = [
    "triton_mxfp8_grouped_mm",
    "triton_mxfp8_wgrad",
    "mxfp8_grouped_mm_to_mx",
    "_rocm_mxfp8_available",
    "_mxfp8_available",
]
