"""mxgg_grouped_mm_noalloc: the forward grouped GEMM for callers that cannot
get device memory at call time (no workspace, no allocation inside the call).

It must give the same result as mxgg_grouped_mm with a caller workspace, on
consecutive calls that reuse its one static scratch array, and refuse
problems whose scratch would not fit in that array.  This file is collected
last so a failure here leaves every other test's result in place.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import O, f32, offsets

pytestmark = pytest.mark.gpu

REL_BF16 = 1e-3   # the bf16-output tolerance the other GEMM tests use


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_matches_workspace_entry_point():
    import utils
    from mxgg import _lib
    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    E, M, N, K = 4, 1536, 768, 1024
    g = torch.Generator().manual_seed(21)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    B = torch.randn(E, N, K, generator=g).to(torch.bfloat16).cuda()
    a_s, a_q = utils.to_mx(A)
    b_s, b_q = utils.to_mx(B)
    offs = torch.tensor(offsets(E, M, 32, seed=21), dtype=torch.int32, device="cuda")

    # the existing entry point, with a workspace from the caller
    ref = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    wsb = lib.mxgg_grouped_mm_workspace_size(M, N, K, E)
    ws = torch.empty(wsb + 256, dtype=torch.uint8, device="cuda")
    wp = ctypes.c_void_p(ws.data_ptr() + (-ws.data_ptr()) % 256)
    _lib.check(lib.mxgg_grouped_mm(_vp(a_q), _vp(b_q), _vp(a_s), _vp(b_s), _vp(offs), M, N, K, E, _vp(ref),
                                   _lib.DTYPE_BF16, wp, wsb, stream), "mxgg_grouped_mm")
    torch.cuda.synchronize()
    ref_np = f32(ref)

    # two calls in a row through the no-allocation entry point
    for _ in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        _lib.check(lib.mxgg_grouped_mm_noalloc(_vp(a_q), _vp(b_q), _vp(a_s), _vp(b_s), _vp(offs), M, N, K, E,
                                               _vp(out), _lib.DTYPE_BF16, stream), "mxgg_grouped_mm_noalloc")
        torch.cuda.synchronize()
        got = f32(out)
        assert np.isfinite(got).all()
        assert O.rel_l2(got, ref_np) <= REL_BF16


def test_noalloc_rejects_oversized_problem():
    from mxgg import _lib
    lib = _lib.load()
    # 64 experts of 8192 x 8192: the packed scales alone exceed the static array
    E, M, N, K = 64, 16640, 8192, 8192
    assert lib.mxgg_grouped_mm_workspace_size(M, N, K, E) > (32 << 20)
    dummy = ctypes.c_void_p(256)
    rc = lib.mxgg_grouped_mm_noalloc(dummy, dummy, dummy, dummy, dummy, M, N, K, E, dummy, _lib.DTYPE_BF16,
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 3
    assert "static array" in lib.mxgg_last_error().decode()
