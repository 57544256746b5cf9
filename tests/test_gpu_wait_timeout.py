"""The GEMM's failure path: a bounded device-side wait that runs out.

The expert-parallel forward loads a segment's rows only once that segment's
source rank has raised its flag.  Here the flag is a local device word that
nothing ever sets, with the wait limit cut to 20 ms: the call must come back,
the device status word must carry bit 128 (a source's rows never arrived),
and the context must stay usable -- the next ordinary GEMM, after the status
is cleared and the limit restored, matches the oracle.  No fault, no hang:
the wait gives up by design.
"""
import ctypes
import time

import numpy as np
import pytest
import torch

from helpers import O, bf16_round, f32, u8

pytestmark = pytest.mark.gpu

ERR_SOURCE_WAIT = 128


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def test_source_wait_runs_out_and_the_next_call_is_correct():
    import utils
    from mxgg import _lib
    lib = _lib.load()
    stream = torch.cuda.current_stream()
    sv = ctypes.c_void_p(stream.cuda_stream)
    E, M, N, K = 2, 512, 256, 256
    g = torch.Generator().manual_seed(5)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    B = torch.randn(E, N, K, generator=g).to(torch.bfloat16).cuda()
    a_s, a_q = utils.to_mx(A)
    b_s, b_q = utils.to_mx(B)
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device="cuda")  # noqa: E731
    seg_offs, seg_expert = i32([256, 512]), i32([0, 1])
    seg_dst, seg_dst_row, seg_src = i32([0, 0]), i32([0, 256]), i32([1, 1])   # rows "from rank 1"
    out = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")
    other = torch.zeros(M, N, dtype=torch.bfloat16, device="cuda")            # destination 1 (unused)
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")                  # nobody raises them
    outs = (ctypes.c_void_p * 2)(out.data_ptr(), other.data_ptr())
    rows = (ctypes.c_int64 * 2)(M, 0)
    wsb = lib.mxgg_grouped_mm_segments_workspace_size(M, N, K, 2, E)
    ws = torch.empty(wsb + 256, dtype=torch.uint8, device="cuda")
    wp = ctypes.c_void_p(ws.data_ptr() + (-ws.data_ptr()) % 256)
    _lib.device_status(clear=True)
    _lib.set_wait_limit(20_000_000)          # 20 ms
    try:
        assert _lib.wait_limit() == 20_000_000
        t0 = time.perf_counter()
        _lib.check(lib.mxgg_grouped_mm_ep(_vp(a_q), _vp(b_q), _vp(a_s), _vp(b_s), _vp(seg_offs), _vp(seg_expert),
                                          _vp(seg_dst), _vp(seg_dst_row), M, N, K, 2, E, _lib.FMT_E4M3, outs, rows,
                                          None, 2, 0, None, _vp(flags), 1, _vp(seg_src), None, 0, -1, 0, None, None,
                                          _lib.DTYPE_BF16, wp, wsb, sv), "mxgg_grouped_mm_ep")
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
        status = _lib.device_status(clear=True)
    finally:
        _lib.set_wait_limit(0)
    assert status & ERR_SOURCE_WAIT, f"status {status:#x}"
    assert elapsed < 5.0, f"the call took {elapsed:.2f} s"
    assert _lib.wait_limit() == 1_000_000_000
    # the context is still usable: an ordinary call is correct and raises nothing
    offs = i32([256, 512])
    import kernels
    res = kernels.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, offs)
    torch.cuda.synchronize()
    assert _lib.device_status(clear=True) == 0
    ref = O.grouped_mm(u8(a_q), u8(a_s), u8(b_q), u8(b_s), np.array([256, 512]), acc=np.float32)
    assert O.rel_l2(f32(res), bf16_round(ref)) <= 1e-3

