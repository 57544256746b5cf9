"""Forward / dgrad MXFP8 grouped GEMM: ``triton_mxfp8_grouped_mm``.

Same signature and argument meaning as the reference
(``kernels/forward.py:461-606``): ``output[g] = input_act[group_g] @
weight[g]^T`` per expert group over jagged token offsets.  The dgrad pass uses
the same call with ``input_act = grad_output`` quantised along N and
``weight = W^T`` (E, K, N) quantised along N.

The Triton/AMD tuning keywords (BLOCK_*, GROUP_M, XCD_SWIZZLE, num_warps,
num_stages, matrix_instr_nonkdim, waves_per_eu, kpack, cache hints) are
accepted for drop-in compatibility (the reference's tuner passes them,
tune_worker.py:87-91) and ignored: the sm_100a kernel picks its own tiles,
or takes them from a table ``mxgg.tune`` measured on B200 (the counterpart
of the reference's ``_BEST_CFGS`` / ``_pick_config``, forward.py:399-459).
"""

import torch

import mxgg
from mxgg import tune as _tune

from ._common import _UNAVAILABLE_MSG, _mxfp8_available, _scale_layout


def triton_mxfp8_grouped_mm(
    input_act: torch.Tensor,
    weight: torch.Tensor,
    input_act_scales: torch.Tensor,
    weight_scales: torch.Tensor,
    group_end_offsets: torch.Tensor,
    out_dtype: torch.dtype = torch.bfloat16,
    BLOCK_M: int = None,
    BLOCK_N: int = None,
    BLOCK_K: int = None,
    GROUP_M: int = None,
    XCD_SWIZZLE: int = None,
    num_warps: int = None,
    num_stages: int = None,
    matrix_instr_nonkdim: int = None,
    waves_per_eu: int = None,
    kpack: int = 1,
    w_cache_modifier: str = None,
    x_evict_policy: str = None,
    scale_layout: str = "row_major",
) -> torch.Tensor:
    """MXFP8 grouped GEMM: ``output[g] = input_act[group_g] @ weight[g]^T``.

    Args:
        input_act: ``(M, K)`` float8_e4m3fn, row-major.
        weight: ``(E, N, K)`` float8_e4m3fn, row-major.
        input_act_scales: ``(M, K//32)`` e8m0 (uint8 or float8_e8m0fnu).
        weight_scales: ``(E, N, K//32)`` e8m0.
        group_end_offsets: ``(E,)`` int32 cumulative token counts per expert.

    Returns ``(M, N)`` of ``out_dtype``; rows at or past ``group_end_offsets[-1]``
    are left unwritten, like the reference (forward.py:583).

    ``weight`` may also be MXFP4: ``(E, N, K//2)`` ``float4_e2m1fn_x2`` (two
    e2m1 values per byte, from ``utils.to_mx(w, elem_dtype=torch.float4_e2m1fn_x2)``)
    with the same ``(E, N, K//32)`` scales; the product runs on the same
    block-scaled tensor-core path.  The reference has no MXFP4 path.

    ``scale_layout`` (not in the reference): ``"row_major"`` takes the
    reference's scale matrices, re-laid on the GPU for the tensor cores on
    every call (one extra launch); ``"blocked"`` takes them already in that
    layout, as ``utils.to_mx_grouped_blocked`` writes them (activation scales
    per group of ``group_end_offsets``, weight scales per expert), and the
    call is the GEMM launch alone.  The results are bit-identical.
    """
    if not _mxfp8_available:
        raise NotImplementedError(_UNAVAILABLE_MSG)
    layout = _scale_layout(scale_layout)
    M, K = input_act.shape
    E, N, K2 = weight.shape
    if weight.dtype == torch.float4_e2m1fn_x2:
        assert K == 2 * K2, f"K mismatch: A={K}, B={2 * K2} (e2m1 packed)"
        experts = torch.arange(E, dtype=torch.int32, device=weight.device)
        return mxgg.ops.grouped_mm_segments(input_act, weight, input_act_scales, weight_scales,
                                            group_end_offsets, experts, out_dtype,
                                            _tune.call_config(_tune.pick("fwd", E, N, K)), layout)
    assert K == K2, f"K mismatch: A={K}, B={K2}"
    # a tuned config for this call shape (mxgg.tune), passed with the call;
    # None: the library's choice
    return mxgg.ops.grouped_mm(input_act, weight, input_act_scales, weight_scales, group_end_offsets, out_dtype,
                               _tune.call_config(_tune.pick("fwd", E, N, K)), layout)


def mxfp8_grouped_mm_to_mx(
    input_act: torch.Tensor,
    weight: torch.Tensor,
    input_act_scales: torch.Tensor,
    weight_scales: torch.Tensor,
    group_end_offsets: torch.Tensor,
    out_dtype: torch.dtype = torch.bfloat16,
    return_output: bool = False,
    dim1: bool = False,
):
    """``to_mx(triton_mxfp8_grouped_mm(...))`` in one kernel: the next
    layer's MXFP8 operand written by the GEMM's epilogue.

    Same arguments as ``triton_mxfp8_grouped_mm`` (``out_dtype`` bf16 or
    f16, ``N % 32 == 0``).  Returns ``(scales (M, N//32) uint8, data (M, N)
    float8_e4m3fn)`` -- ``to_mx``'s order -- bit for bit what ``to_mx`` gives
    for the ``out_dtype`` output, which is never written to HBM unless
    ``return_output`` (then ``(scales, data, output)``).  With ``dim1`` the
    epilogue also writes ``utils.to_mx_dim1`` of the output -- the transpose
    quantised along tokens, ``(scales_t (N, M//32), data_t (N, M))``, the
    operand layout of the next ``triton_mxfp8_wgrad`` -- appended after
    ``data``; it needs ``M % 32 == 0`` and group ends on multiples of 32.  A
    group off that grid sets device status bit 256 and its transposed blocks
    are left unwritten (the buffers are not zeroed), so a caller whose offsets
    may be off the grid must check ``mxgg.device_status()`` before using
    them.  Rows at or past
    ``group_end_offsets[-1]`` are left unwritten.  The reference runs the GEMM
    (kernels/forward.py:461-606) and ``to_mx`` (utils.py:67-105) separately.
    """
    if not _mxfp8_available:
        raise NotImplementedError(_UNAVAILABLE_MSG)
    M, K = input_act.shape
    E, N, K2 = weight.shape
    packed = weight.dtype == torch.float4_e2m1fn_x2
    assert K == (2 * K2 if packed else K2), f"K mismatch: A={K}, B={2 * K2 if packed else K2}"
    s, q, st, qt, out = mxgg.ops.grouped_mm_mx(input_act, weight, input_act_scales, weight_scales,
                                               group_end_offsets, None, out_dtype, return_output, True, dim1,
                                               _tune.call_config(_tune.pick("fwd", E, N, K)))
    res = (s, q, st, qt) if dim1 else (s, q)
    return res + (out,) if return_output else res
