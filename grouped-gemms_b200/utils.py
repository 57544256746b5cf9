"""Helpers with the reference's ``utils.py`` names (drop-in surface).

* ``to_mx`` -- MXFP8 quantiser, bit-exact with the reference's FLOOR-mode
  ``utils.to_mx`` (utils.py:67-105), run by the sm_100a quantise kernel.
* ``to_mx_dim1`` -- ``to_mx(x.t().contiguous())`` fused into one pass: the
  operand layout of ``triton_mxfp8_wgrad`` (scales along tokens).
* ``generate_jagged_offs`` -- same seeded draw as utils.py:35-50.
* ``benchmark_cuda_function_in_microseconds`` -- median device time with an
  L2 flush between runs (the reference delegates to triton's do_bench).
"""

import random
from typing import Callable

import torch

import mxgg
from mxgg import _lib


def _check_to_mx_args(data: torch.Tensor, elem_dtype, block_size: int) -> None:
    assert elem_dtype in (torch.float8_e4m3fn, torch.float4_e2m1fn_x2), "only e4m3fn (and e2m1 weights) supported here"
    assert data.shape[-1] % block_size == 0, (
        f"last dim {data.shape[-1]} must be divisible by block_size {block_size}"
    )
    if block_size != 32:
        raise NotImplementedError("the sm_100a quantiser implements the MX block size 32 only")


def to_mx(data: torch.Tensor, elem_dtype=torch.float8_e4m3fn, block_size: int = 32):
    """Quantise ``data`` to MXFP8 along the last dim.

    Returns ``(scales_e8m0_as_uint8, data_fp8)`` -- scales first, as in the
    reference (utils.py:67-105).  ``data`` must be a CUDA bf16/fp16/fp32
    tensor; any leading shape is kept.
    """
    _check_to_mx_args(data, elem_dtype, block_size)
    orig_shape = data.shape
    x2 = data.reshape(-1, orig_shape[-1])
    scale_shape = list(orig_shape)
    scale_shape[-1] = orig_shape[-1] // block_size
    if elem_dtype is torch.float4_e2m1fn_x2:
        # MXFP4 (no reference counterpart): FLOOR scaling with emax 2, two
        # e2m1 values per byte, element 2i in the low nibble
        s, q = mxgg.ops.to_mx_fp4(x2, _lib.SCALE_ROW_MAJOR)
        q_shape = list(orig_shape)
        q_shape[-1] = orig_shape[-1] // 2
        return s.reshape(scale_shape), q.reshape(q_shape)
    s, q = mxgg.ops.to_mx(x2, _lib.QUANT_ROWS, _lib.SCALE_ROW_MAJOR)
    return s.reshape(scale_shape), q.reshape(orig_shape)


def to_mx_dim1(data: torch.Tensor, elem_dtype=torch.float8_e4m3fn, block_size: int = 32):
    """``to_mx(data.t().contiguous())`` for a 2-D ``data`` (R, C), in one pass.

    Returns ``(scales (C, R//32), data_fp8 (C, R))``.
    """
    assert data.dim() == 2, "to_mx_dim1 takes a 2-D tensor"
    _check_to_mx_args(data.t(), elem_dtype, block_size)
    return mxgg.ops.to_mx(data, _lib.QUANT_COLS, _lib.SCALE_ROW_MAJOR)


def to_mx_blocked_scales(data: torch.Tensor):
    """``to_mx`` with the scales written in the 128x4 blocked atom layout
    (rows padded to 128, scale columns to 4) that Blackwell block-scaled MMAs
    and ``torch._scaled_mm`` consume.  Returns ``(scales_flat_u8, data_fp8)``.
    """
    assert data.dim() == 2 and data.shape[-1] % 32 == 0
    return mxgg.ops.to_mx(data, _lib.QUANT_ROWS, _lib.SCALE_BLOCKED)


def to_mx_grouped_blocked(data: torch.Tensor, group_end_offsets: torch.Tensor = None):
    """``to_mx`` with the scales written once, in the blocked layout the
    grouped GEMMs read with ``scale_layout="blocked"``: a 2-D ``data`` (M, K)
    with ``group_end_offsets`` is an activation (each group's scale rows start
    a new 128-row slab), a 3-D ``data`` (E, N, K) a weight (each expert's).
    Returns ``(scales, data_fp8)``: the scales as one flat uint8 tensor
    (zero padding), the data in ``data``'s shape.  No reference counterpart.
    """
    if data.dim() == 3:
        E, N, K = data.shape
        s, q = mxgg.ops.to_mx_blocked(data.reshape(E * N, K), None, E)
        return s, q.reshape(E, N, K)
    assert data.dim() == 2 and group_end_offsets is not None, \
        "a 2-D activation needs its group_end_offsets"
    return mxgg.ops.to_mx_blocked(data, group_end_offsets, 0)


def to_mx_dim1_blocked(data: torch.Tensor):
    """``to_mx_dim1`` with the scales in the one-segment blocked layout
    (the weight-gradient operands' layout for ``scale_layout="blocked"``).
    Returns ``(scales flat uint8, data_fp8 (C, R))``.
    """
    assert data.dim() == 2, "to_mx_dim1_blocked takes a 2-D tensor"
    _check_to_mx_args(data.t(), torch.float8_e4m3fn, 32)
    return mxgg.ops.to_mx(data, _lib.QUANT_COLS, _lib.SCALE_BLOCKED)


def generate_jagged_offs(E: int, M: int, multiple_of: int = 32, dtype=torch.int32, device="cuda") -> torch.Tensor:
    """Random sorted cumulative offsets summing to M, each a multiple of
    ``multiple_of``; the last value is M.  Same draw as utils.py:35-50
    (Python ``random.sample``: seed ``random`` for reproducibility).
    """
    if M % multiple_of != 0:
        raise ValueError(f"M must be divisible by {multiple_of}")
    possible_values = list(range(multiple_of, M + 1, multiple_of))
    if E > len(possible_values):
        raise ValueError("E cannot be larger than the number of possible values")
    selected = sorted(random.sample(possible_values[:-1], E - 1) + [M])
    return torch.tensor(selected, dtype=dtype, device=device)


_flush_buf = {}


def flush_l2(device=None) -> None:
    """Overwrite a 512 MiB buffer so the next kernel starts with a cold L2 (126 MB)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    buf = _flush_buf.get(dev)
    if buf is None:
        buf = torch.empty(512 * 1024 * 1024 // 4, dtype=torch.int32, device=dev)
        _flush_buf[dev] = buf
    buf.zero_()


def benchmark_cuda_function_in_microseconds(fn: Callable, *args, warmup: int = 5, reps: int = 50,
                                            **kwargs) -> float:
    """Median device runtime of ``fn(*args, **kwargs)`` in microseconds.

    Each timed call is preceded by an L2 flush and bracketed by CUDA events on
    the current stream.
    """
    for _ in range(warmup):
        fn(*args, **kwargs)
    torch.cuda.synchronize()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(reps)]
    for i in range(reps):
        flush_l2()
        starts[i].record()
        fn(*args, **kwargs)
        ends[i].record()
    torch.cuda.synchronize()
    times = sorted(s.elapsed_time(e) * 1e3 for s, e in zip(starts, ends))
    return times[len(times) // 2]


def is_MI350() -> bool:
    """The reference's gfx950 probe (utils.py:108-115); always False on NVIDIA."""
    if getattr(torch.version, "hip", None) is None:
        return False
    try:
        arch = torch.cuda.get_device_properties(0).gcnArchName
    except Exception:
        return False
    return "gfx950" in arch


def is_sm100() -> bool:
    """True on a compute-capability 10.0 (B200-class) device."""
    return torch.cuda.is_available() and torch.cuda.get_device_capability() == (10, 0)
