"""torch.library custom ops over the mxgg C ABI.

``mxgg::to_mx``, ``mxgg::grouped_mm`` and ``mxgg::wgrad`` enqueue the sm_100a
kernels on the current CUDA stream through ctypes; nothing here synchronises,
so the ops are safe inside CUDA graphs.  Each op has a fake (meta) kernel so
``torch.compile`` can trace callers.  There is no CPU implementation: CPU
tensors raise.
"""

import ctypes
from typing import List, Optional, Tuple

import torch
from torch import Tensor
from torch.utils._python_dispatch import _get_current_dispatch_mode

from . import _lib

_OUT_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float16: _lib.DTYPE_F16, torch.float32: _lib.DTYPE_F32}
_IN_DTYPES = dict(_OUT_DTYPES)


def _ptr(t: Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _require_cuda(*ts: Tensor, what: str) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError(f"{what}: mxgg runs only on CUDA (sm_100a) tensors; got a {t.device} tensor")


def _workspace(nbytes: int, device: torch.device) -> Tensor:
    """Scratch for one GEMM call from torch's caching allocator (256-byte aligned)."""
    if nbytes < 0:
        raise ValueError("mxgg: invalid GEMM sizes")
    buf = torch.empty(nbytes + 256, dtype=torch.uint8, device=device)
    off = (-buf.data_ptr()) % 256
    return buf[off:off + nbytes]


def b_format_of(b: Tensor) -> int:
    """MXGG_FMT_E2M1 for packed MXFP4 weights (float4_e2m1fn_x2), else e4m3."""
    return _lib.FMT_E2M1 if b.dtype == torch.float4_e2m1fn_x2 else _lib.FMT_E4M3


def as_u8(t: Tensor) -> Tensor:
    """Scales may be uint8 or float8_e8m0fnu (reference forward.py:534-535)."""
    return t if t.dtype == torch.uint8 else t.view(torch.uint8)


def _eager(args) -> bool:
    """True when a call may run its implementation directly instead of going
    through the torch.library dispatcher (which costs ~15 us of host time per
    call): eager mode, no dispatch mode active (FakeTensor tracing, flop
    counters), and plain tensors that need no autograd.  Anything else takes
    the registered op, so torch.compile and tensor subclasses see it."""
    if torch.compiler.is_compiling() or _get_current_dispatch_mode() is not None:
        return False
    for t in args:
        if isinstance(t, Tensor) and (type(t) is not Tensor or t.requires_grad):
            return False
    return True


def _fast(op, impl):
    """`op`'s eager fast path: `impl` directly when `_eager` allows, else `op`."""
    def call(*args):
        return impl(*args) if _eager(args) else op(*args)
    call.__name__ = getattr(impl, "__name__", "call").lstrip("_").replace("_impl", "")
    call.__doc__ = impl.__doc__
    return call


# --------------------------------------------------------------------- to_mx
def _to_mx_impl(x: Tensor, mode: int, scale_layout: int) -> Tuple[Tensor, Tensor]:
    _require_cuda(x, what="mxgg::to_mx")
    if x.dtype not in _IN_DTYPES:
        raise TypeError(f"mxgg::to_mx: unsupported input dtype {x.dtype}")
    x = x.contiguous()
    R, C = x.shape
    lib = _lib.load()
    with torch.cuda.device(x.device):
        if mode == _lib.QUANT_ROWS:
            q = torch.empty((R, C), dtype=torch.float8_e4m3fn, device=x.device)
            sr, sc = R, C // 32
        else:
            q = torch.empty((C, R), dtype=torch.float8_e4m3fn, device=x.device)
            sr, sc = C, R // 32
        if scale_layout == _lib.SCALE_BLOCKED:
            s = torch.zeros(((sr + 127) // 128 * 128) * ((sc + 3) // 4 * 4), dtype=torch.uint8, device=x.device)
        else:
            s = torch.empty((sr, sc), dtype=torch.uint8, device=x.device)
        _lib.check(lib.mxgg_quantize_mx(_ptr(x), _IN_DTYPES[x.dtype], R, C, _ptr(q), _ptr(s), mode,
                                        scale_layout, _stream(x.device)), "mxgg_quantize_mx")
    return s, q


to_mx_op = torch.library.custom_op("mxgg::to_mx", _to_mx_impl, mutates_args=())
to_mx = _fast(to_mx_op, _to_mx_impl)


@to_mx_op.register_fake
def _(x, mode, scale_layout):
    R, C = x.shape
    if mode == _lib.QUANT_ROWS:
        q = x.new_empty((R, C), dtype=torch.float8_e4m3fn)
        sr, sc = R, C // 32
    else:
        q = x.new_empty((C, R), dtype=torch.float8_e4m3fn)
        sr, sc = C, R // 32
    if scale_layout == _lib.SCALE_BLOCKED:
        s = x.new_empty(((sr + 127) // 128 * 128) * ((sc + 3) // 4 * 4), dtype=torch.uint8)
    else:
        s = x.new_empty((sr, sc), dtype=torch.uint8)
    return s, q


def _to_mx_blocked_impl(x: Tensor, offs: Optional[Tensor], n_segments: int) -> Tuple[Tensor, Tensor]:
    """to_mx along the last dim of a 2-D x, with the scales in the segmented
    blocked layout the grouped GEMM reads when called with SCALE_BLOCKED:
    segments are the groups (offs, cumulative row ends) or, with offs None,
    n_segments equal row blocks (the experts of a flattened (E * N, K)
    weight).  Returns (scales, a flat zero-padded uint8 tensor, q (R, C))."""
    _require_cuda(x, what="mxgg::to_mx_blocked")
    if x.dtype not in _IN_DTYPES:
        raise TypeError(f"mxgg::to_mx_blocked: unsupported input dtype {x.dtype}")
    x = x.contiguous()
    R, C = x.shape
    lib = _lib.load()
    S = offs.shape[0] if offs is not None else int(n_segments)
    if offs is None and (S < 1 or R % S != 0):
        raise ValueError(f"mxgg::to_mx_blocked: {R} rows do not split into {S} equal segments")
    with torch.cuda.device(x.device):
        q = torch.empty((R, C), dtype=torch.float8_e4m3fn, device=x.device)
        s = torch.zeros(max(int(lib.mxgg_blocked_scale_bytes(R, C, S)), 0), dtype=torch.uint8, device=x.device)
        if offs is not None:
            _require_cuda(offs, what="mxgg::to_mx_blocked")
            offs = offs.to(torch.int32).contiguous()
        _lib.check(lib.mxgg_quantize_mx_blocked(_ptr(x), _IN_DTYPES[x.dtype], R, C, _ptr(q), _ptr(s),
                                                _ptr(offs) if offs is not None else None, S,
                                                0 if offs is not None else R // S, _stream(x.device)),
                   "mxgg_quantize_mx_blocked")
    return s, q


to_mx_blocked_op = torch.library.custom_op("mxgg::to_mx_blocked", _to_mx_blocked_impl, mutates_args=())
to_mx_blocked = _fast(to_mx_blocked_op, _to_mx_blocked_impl)


@to_mx_blocked_op.register_fake
def _(x, offs, n_segments):
    R, C = x.shape
    S = offs.shape[0] if offs is not None else int(n_segments)
    nbytes = ((R + 127) // 128 + S - 1) * ((C + 127) // 128) * 512
    return x.new_empty((nbytes,), dtype=torch.uint8), x.new_empty((R, C), dtype=torch.float8_e4m3fn)


def _to_mx_fp4_impl(x: Tensor, scale_layout: int) -> Tuple[Tensor, Tensor]:
    """MXFP4 along the last dim: (scales (R, C/32) u8, q (R, C/2) float4_e2m1fn_x2)."""
    _require_cuda(x, what="mxgg::to_mx_fp4")
    if x.dtype not in _IN_DTYPES:
        raise TypeError(f"mxgg::to_mx_fp4: unsupported input dtype {x.dtype}")
    x = x.contiguous()
    R, C = x.shape
    with torch.cuda.device(x.device):
        q = torch.empty((R, C // 2), dtype=torch.uint8, device=x.device)
        if scale_layout == _lib.SCALE_BLOCKED:
            s = torch.zeros(((R + 127) // 128 * 128) * ((C // 32 + 3) // 4 * 4), dtype=torch.uint8, device=x.device)
        else:
            s = torch.empty((R, C // 32), dtype=torch.uint8, device=x.device)
        _lib.check(_lib.load().mxgg_quantize_mx_fp4(_ptr(x), _IN_DTYPES[x.dtype], R, C, _ptr(q), _ptr(s),
                                                    scale_layout, _stream(x.device)), "mxgg_quantize_mx_fp4")
    return s, q.view(torch.float4_e2m1fn_x2)


to_mx_fp4_op = torch.library.custom_op("mxgg::to_mx_fp4", _to_mx_fp4_impl, mutates_args=())
to_mx_fp4 = _fast(to_mx_fp4_op, _to_mx_fp4_impl)


@to_mx_fp4_op.register_fake
def _(x, scale_layout):
    R, C = x.shape
    q = x.new_empty((R, C // 2), dtype=torch.float4_e2m1fn_x2)
    if scale_layout == _lib.SCALE_BLOCKED:
        s = x.new_empty(((R + 127) // 128 * 128) * ((C // 32 + 3) // 4 * 4), dtype=torch.uint8)
    else:
        s = x.new_empty((R, C // 32), dtype=torch.uint8)
    return s, q


# ---------------------------------------------------------------- grouped_mm
def _grouped_mm_impl(a: Tensor, b: Tensor, a_scale: Tensor, b_scale: Tensor, offs: Tensor,
                  out_dtype: torch.dtype, cfg: Optional[List[int]] = None, scale_layout: int = 0) -> Tensor:
    """cfg: this call's (tile_m, tile_n, group_m, schedule, split_max), zeros
    for the process defaults (mxgg_gemm_config); None: all defaults.
    scale_layout: SCALE_ROW_MAJOR (the reference's (rows, K/32) scales) or
    SCALE_BLOCKED (the blocked layout to_mx_blocked writes: A per group, B
    per expert; no re-layout launch)."""
    _require_cuda(a, b, a_scale, b_scale, offs, what="mxgg::grouped_mm")
    if out_dtype not in _OUT_DTYPES:
        raise TypeError(f"mxgg::grouped_mm: unsupported out_dtype {out_dtype}")
    M, K = a.shape
    E, N, _ = b.shape
    a = a.contiguous()
    b = b.contiguous()
    a_scale = as_u8(a_scale).contiguous()
    b_scale = as_u8(b_scale).contiguous()
    offs = offs.to(torch.int32).contiguous()
    out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    lib = _lib.load()
    ws = _workspace(lib.mxgg_grouped_mm_workspace_size(M, N, K, E), a.device)
    with torch.cuda.device(a.device):
        _lib.check(lib.mxgg_grouped_mm_cfg(_ptr(a), _ptr(b), _ptr(a_scale), _ptr(b_scale), _ptr(offs),
                                           M, N, K, E, _ptr(out), _OUT_DTYPES[out_dtype], _lib.gemm_config(cfg, scale_layout),
                                           _ptr(ws), ws.numel(), _stream(a.device)), "mxgg_grouped_mm")
    return out


grouped_mm_op = torch.library.custom_op("mxgg::grouped_mm", _grouped_mm_impl, mutates_args=())
grouped_mm = _fast(grouped_mm_op, _grouped_mm_impl)


@grouped_mm_op.register_fake
def _(a, b, a_scale, b_scale, offs, out_dtype, cfg=None, scale_layout=0):
    return a.new_empty((a.shape[0], b.shape[1]), dtype=out_dtype)


# ------------------------------------------------------- grouped_mm_segments
def _grouped_mm_segments_impl(a: Tensor, b: Tensor, a_scale: Tensor, b_scale: Tensor, seg_offs: Tensor,
                           seg_expert: Tensor, out_dtype: torch.dtype, cfg: Optional[List[int]] = None,
                           scale_layout: int = 0) -> Tensor:
    """Rows of segment s times B[seg_expert[s]]: the layout an expert-parallel
    all-to-all delivers (source-major, then expert)."""
    _require_cuda(a, b, a_scale, b_scale, seg_offs, seg_expert, what="mxgg::grouped_mm_segments")
    if out_dtype not in _OUT_DTYPES:
        raise TypeError(f"mxgg::grouped_mm_segments: unsupported out_dtype {out_dtype}")
    M, K = a.shape
    E, N, _ = b.shape
    b_format = b_format_of(b)
    S = seg_offs.shape[0]
    a = a.contiguous()
    b = b.contiguous()
    a_scale = as_u8(a_scale).contiguous()
    b_scale = as_u8(b_scale).contiguous()
    seg_offs = seg_offs.to(torch.int32).contiguous()
    seg_expert = seg_expert.to(torch.int32).contiguous()
    out = torch.empty((M, N), dtype=out_dtype, device=a.device)
    lib = _lib.load()
    ws = _workspace(lib.mxgg_grouped_mm_segments_workspace_size(M, N, K, S, E), a.device)
    with torch.cuda.device(a.device):
        _lib.check(lib.mxgg_grouped_mm_segments_cfg(_ptr(a), _ptr(b), _ptr(a_scale), _ptr(b_scale),
                                                    _ptr(seg_offs), _ptr(seg_expert), M, N, K, S, E, b_format,
                                                    _ptr(out), _OUT_DTYPES[out_dtype], _lib.gemm_config(cfg, scale_layout),
                                                    _ptr(ws), ws.numel(), _stream(a.device)),
                   "mxgg_grouped_mm_segments")
    return out


grouped_mm_segments_op = torch.library.custom_op("mxgg::grouped_mm_segments", _grouped_mm_segments_impl,
                                                 mutates_args=())
grouped_mm_segments = _fast(grouped_mm_segments_op, _grouped_mm_segments_impl)


@grouped_mm_segments_op.register_fake
def _(a, b, a_scale, b_scale, seg_offs, seg_expert, out_dtype, cfg=None, scale_layout=0):
    return a.new_empty((a.shape[0], b.shape[1]), dtype=out_dtype)


def _grouped_mm_mx_impl(a: Tensor, b: Tensor, a_scale: Tensor, b_scale: Tensor, seg_offs: Tensor,
                     seg_expert: Optional[Tensor], out_dtype: torch.dtype, keep_out: bool, rows: bool = True,
                     cols: bool = False, cfg: Optional[List[int]] = None,
                     scale_layout: int = 0) -> Tuple[Tensor, Tensor, Tensor, Tensor, Tensor]:
    """The forward (segments as in grouped_mm_segments_op; seg_expert None:
    segment s uses expert s) with MX quantisation of its output fused into
    the epilogue.  Returns (scales, data, scales_t, data_t, out):
      rows: to_mx(out)      -- scales (M, N//32) uint8, data (M, N) e4m3;
      cols: to_mx(out.t())  -- scales_t (N, M//32), data_t (N, M) (M % 32 == 0,
            segments on the 32-row grid);
      keep_out: out (M, N) of out_dtype.
    Parts not asked for come back as empty tensors."""
    _require_cuda(a, b, a_scale, b_scale, seg_offs, what="mxgg::grouped_mm_mx")
    if out_dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"mxgg::grouped_mm_mx: out_dtype must be bf16 or f16, got {out_dtype}")
    M, K = a.shape
    E, N, _ = b.shape
    if N % 32 != 0:
        raise ValueError(f"mxgg::grouped_mm_mx: N={N} must be a multiple of 32")
    if not (rows or cols):
        raise ValueError("mxgg::grouped_mm_mx: ask for rows and/or cols")
    if cols and M % 32 != 0:
        raise ValueError(f"mxgg::grouped_mm_mx: the transposed output needs M % 32 == 0 (M={M})")
    b_format = b_format_of(b)
    S = seg_offs.shape[0]
    a = a.contiguous()
    b = b.contiguous()
    a_scale = as_u8(a_scale).contiguous()
    b_scale = as_u8(b_scale).contiguous()
    seg_offs = seg_offs.to(torch.int32).contiguous()
    if seg_expert is not None:
        _require_cuda(seg_expert, what="mxgg::grouped_mm_mx")
        seg_expert = seg_expert.to(torch.int32).contiguous()
    elif S != E:
        raise ValueError(f"mxgg::grouped_mm_mx: {S} segments need a segment -> expert map for {E} experts")
    dev = a.device
    out = torch.empty((M, N) if keep_out else (0,), dtype=out_dtype, device=dev)
    q = torch.empty((M, N) if rows else (0,), dtype=torch.float8_e4m3fn, device=dev)
    s = torch.empty((M, N // 32) if rows else (0,), dtype=torch.uint8, device=dev)
    qt = torch.empty((N, M) if cols else (0,), dtype=torch.float8_e4m3fn, device=dev)
    st = torch.empty((N, M // 32) if cols else (0,), dtype=torch.uint8, device=dev)
    opt = lambda t, on: _ptr(t) if on else None  # noqa: E731
    lib = _lib.load()
    ws = _workspace(lib.mxgg_grouped_mm_segments_workspace_size(M, N, K, S, E), dev)
    with torch.cuda.device(dev):
        _lib.check(lib.mxgg_grouped_mm_mx_cfg(_ptr(a), _ptr(b), _ptr(a_scale), _ptr(b_scale), _ptr(seg_offs),
                                              _ptr(seg_expert) if seg_expert is not None else None, M, N, K, S, E,
                                              b_format, opt(out, keep_out), _OUT_DTYPES[out_dtype], opt(q, rows),
                                              opt(s, rows), opt(qt, cols), opt(st, cols), _lib.gemm_config(cfg, scale_layout),
                                              _ptr(ws), ws.numel(), _stream(dev)),
                   "mxgg_grouped_mm_mx")
    return s, q, st, qt, out


grouped_mm_mx_op = torch.library.custom_op("mxgg::grouped_mm_mx", _grouped_mm_mx_impl, mutates_args=())
grouped_mm_mx = _fast(grouped_mm_mx_op, _grouped_mm_mx_impl)


@grouped_mm_mx_op.register_fake
def _(a, b, a_scale, b_scale, seg_offs, seg_expert, out_dtype, keep_out, rows=True, cols=False, cfg=None,
      scale_layout=0):
    M, N = a.shape[0], b.shape[1]
    e = lambda shape, on, dt: a.new_empty(shape if on else (0,), dtype=dt)  # noqa: E731
    return (e((M, N // 32), rows, torch.uint8), e((M, N), rows, torch.float8_e4m3fn),
            e((N, M // 32), cols, torch.uint8), e((N, M), cols, torch.float8_e4m3fn),
            e((M, N), keep_out, out_dtype))


# --------------------------------------------------------------------- wgrad
def _wgrad_impl(go_t: Tensor, go_scale: Tensor, ia_t: Tensor, ia_scale: Tensor, offs: Tensor,
             out_dtype: torch.dtype, cfg: Optional[List[int]] = None, scale_layout: int = 0) -> Tensor:
    """scale_layout SCALE_BLOCKED: go_scale / ia_scale in the one-segment
    blocked layout (to_mx_dim1 with blocked scales)."""
    _require_cuda(go_t, go_scale, ia_t, ia_scale, offs, what="mxgg::wgrad")
    if out_dtype not in _OUT_DTYPES:
        raise TypeError(f"mxgg::wgrad: unsupported out_dtype {out_dtype}")
    out = torch.empty((offs.shape[0], go_t.shape[0], ia_t.shape[0]), dtype=out_dtype, device=go_t.device)
    wgrad_into(go_t, go_scale, ia_t, ia_scale, offs, out, cfg, scale_layout)
    return out


def wgrad_into(go_t: Tensor, go_scale: Tensor, ia_t: Tensor, ia_scale: Tensor, offs: Tensor, out: Tensor,
               cfg: Optional[List[int]] = None, scale_layout: int = 0) -> Tensor:
    """The weight gradient written into an existing contiguous (E, N, K)
    tensor of any output dtype (for example a buffer peers can read, which
    the replicas of an expert then sum in place); returns `out`."""
    _require_cuda(go_t, go_scale, ia_t, ia_scale, offs, out, what="mxgg::wgrad")
    if out.dtype not in _OUT_DTYPES:
        raise TypeError(f"mxgg::wgrad: unsupported out dtype {out.dtype}")
    N, M = go_t.shape
    K = ia_t.shape[0]
    E = offs.shape[0]
    if out.shape != (E, N, K) or not out.is_contiguous():
        raise ValueError(f"mxgg::wgrad: out must be a contiguous ({E}, {N}, {K}) tensor")
    go_t = go_t.contiguous()
    ia_t = ia_t.contiguous()
    go_scale = as_u8(go_scale).contiguous()
    ia_scale = as_u8(ia_scale).contiguous()
    offs = offs.to(torch.int32).contiguous()
    lib = _lib.load()
    ws = _workspace(lib.mxgg_wgrad_workspace_size(N, K, M, E), go_t.device)
    with torch.cuda.device(go_t.device):
        _lib.check(lib.mxgg_wgrad_cfg(_ptr(go_t), _ptr(go_scale), _ptr(ia_t), _ptr(ia_scale), _ptr(offs),
                                      N, K, M, E, _ptr(out), _OUT_DTYPES[out.dtype], _lib.gemm_config(cfg, scale_layout),
                                      _ptr(ws), ws.numel(), _stream(go_t.device)), "mxgg_wgrad")
    return out


wgrad_op = torch.library.custom_op("mxgg::wgrad", _wgrad_impl, mutates_args=())
wgrad = _fast(wgrad_op, _wgrad_impl)


@wgrad_op.register_fake
def _(go_t, go_scale, ia_t, ia_scale, offs, out_dtype, cfg=None, scale_layout=0):
    return go_t.new_empty((offs.shape[0], go_t.shape[0], ia_t.shape[0]), dtype=out_dtype)


def _wgrad_accumulate_impl(go_t: Tensor, go_scale: Tensor, ia_t: Tensor, ia_scale: Tensor, offs: Tensor,
                        out: Tensor, cfg: Optional[List[int]] = None, scale_layout: int = 0) -> None:
    """out[g] += the group's weight gradient, in place (fp32 out)."""
    _require_cuda(go_t, go_scale, ia_t, ia_scale, offs, out, what="mxgg::wgrad_accumulate_")
    N, M = go_t.shape
    K = ia_t.shape[0]
    E = offs.shape[0]
    if out.dtype != torch.float32 or out.shape != (E, N, K) or not out.is_contiguous():
        raise ValueError(f"mxgg::wgrad_accumulate_: out must be a contiguous fp32 ({E}, {N}, {K}) tensor")
    go_t = go_t.contiguous()
    ia_t = ia_t.contiguous()
    go_scale = as_u8(go_scale).contiguous()
    ia_scale = as_u8(ia_scale).contiguous()
    offs = offs.to(torch.int32).contiguous()
    lib = _lib.load()
    ws = _workspace(lib.mxgg_wgrad_workspace_size(N, K, M, E), go_t.device)
    with torch.cuda.device(go_t.device):
        _lib.check(lib.mxgg_wgrad_accumulate_cfg(_ptr(go_t), _ptr(go_scale), _ptr(ia_t), _ptr(ia_scale),
                                                 _ptr(offs), N, K, M, E, _ptr(out), _lib.gemm_config(cfg, scale_layout),
                                                 _ptr(ws), ws.numel(), _stream(go_t.device)),
                   "mxgg_wgrad_accumulate")


wgrad_accumulate_op = torch.library.custom_op("mxgg::wgrad_accumulate_", _wgrad_accumulate_impl,
                                              mutates_args=("out",))
wgrad_accumulate = _fast(wgrad_accumulate_op, _wgrad_accumulate_impl)


@wgrad_accumulate_op.register_fake
def _(go_t, go_scale, ia_t, ia_scale, offs, out, cfg=None, scale_layout=0):
    return None


def build_tile_map(offs: Tensor, M: int, block_m: int) -> Tensor:
    """Routing tables in the reference's _build_expt_data layout (forward.py:340-365)."""
    _require_cuda(offs, what="mxgg.build_tile_map")
    offs = offs.to(torch.int32).contiguous()
    E = offs.shape[0]
    n = 2 * E + 1 + (M + block_m - 1) // block_m + max(E - 1, 0)
    out = torch.empty(n, dtype=torch.int32, device=offs.device)
    with torch.cuda.device(offs.device):
        _lib.check(_lib.load().mxgg_build_tile_map(_ptr(offs), E, M, block_m, _ptr(out), _stream(offs.device)),
                   "mxgg_build_tile_map")
    return out
