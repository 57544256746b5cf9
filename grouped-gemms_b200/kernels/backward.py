"""Weight-gradient MXFP8 grouped GEMM: ``triton_mxfp8_wgrad``.

Same signature and argument meaning as the reference
(``kernels/backward.py:217-305``): ``grad_W[g] = grad_output[group_g]^T @
input_act[group_g]`` with both inputs dim1-quantised (scales along tokens).
The reference stores bf16 whatever ``out_dtype`` says (backward.py:103,214);
this implementation honours ``out_dtype`` (bf16, fp16 or fp32).  The Triton
tile keywords are accepted and ignored; a table measured by ``mxgg.tune``
supplies B200 tiles per call shape when one is installed.
"""

import torch

import mxgg
from mxgg import tune as _tune

from ._common import _UNAVAILABLE_MSG, _mxfp8_available, _scale_layout


def triton_mxfp8_wgrad(
    go_t: torch.Tensor,
    go_scale: torch.Tensor,
    ia_t: torch.Tensor,
    ia_scale: torch.Tensor,
    group_end_offsets: torch.Tensor,
    out_dtype: torch.dtype = torch.bfloat16,
    BLOCK_N: int = 256,
    BLOCK_K: int = 256,
    BLOCK_M: int = 64,
    num_warps: int = 8,
    num_stages: int = 2,
    out: torch.Tensor = None,
    scale_layout: str = "row_major",
) -> torch.Tensor:
    """MXFP8 weight gradient: ``grad_W[g] = grad_output[group_g]^T @ input_act[group_g]``.

    Args:
        go_t: ``(N, M)`` float8_e4m3fn, with ``go_scale`` ``(N, M//32)``.
        ia_t: ``(K, M)`` float8_e4m3fn, with ``ia_scale`` ``(K, M//32)``.
        group_end_offsets: ``(E,)`` int32, multiples of 32.

    Returns ``(E, N, K)`` of ``out_dtype``; empty groups give zeros.

    ``out`` (not in the reference): an existing fp32 ``(E, N, K)`` gradient
    buffer to accumulate into (``out += grad_W``, one deterministic add per
    element); it is returned.

    ``scale_layout`` (not in the reference): ``"blocked"`` takes both scale
    tensors in the blocked layout ``utils.to_mx_dim1_blocked`` writes (one
    re-layout launch fewer; bit-identical results).
    """
    if not _mxfp8_available:
        raise NotImplementedError(_UNAVAILABLE_MSG)
    layout = _scale_layout(scale_layout)
    # a tuned config for this call shape (mxgg.tune), passed with the call
    cfg = _tune.call_config(_tune.pick("wgrad", group_end_offsets.shape[0], go_t.shape[0], ia_t.shape[0]))
    if out is not None:
        mxgg.ops.wgrad_accumulate(go_t, go_scale, ia_t, ia_scale, group_end_offsets, out, cfg, layout)
        return out
    return mxgg.ops.wgrad(go_t, go_scale, ia_t, ia_scale, group_end_offsets, out_dtype, cfg, layout)
