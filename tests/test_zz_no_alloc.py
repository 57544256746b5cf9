"""mxgg_grouped_mm_noalloc: the forward grouped GEMM for callers that cannot
get device memory at call time (no workspace, no allocation inside the call).

Both calls run the same kernel with the same schedule, so the no-allocation
entry point must return exactly what mxgg_grouped_mm returns with a caller
workspace, on consecutive calls that reuse its one static scratch array; the
result is also checked against the oracle.  A problem whose split-tail
partial tiles do not fit beside its packed scales runs whole tiles and must
equal mxgg_grouped_mm with the whole-tile schedule.  Problems whose packed
scales alone exceed the array are refused.  This file is collected last so a
failure here leaves every other test's result in place.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import O, bf16_round, f32, offsets, u8

pytestmark = pytest.mark.gpu

REL_BF16 = 1e-3   # the bf16-output tolerance of the other GEMM tests (oracle rounded to bf16)
SCRATCH = 32 << 20


def _vp(t):
    return ctypes.c_void_p(t.data_ptr())


def _operands(E, M, N, K, seed):
    import utils
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    B = torch.randn(E, N, K, generator=g).to(torch.bfloat16).cuda()
    a_s, a_q = utils.to_mx(A)
    b_s, b_q = utils.to_mx(B)
    offs = torch.tensor(offsets(E, M, 32, seed=seed), dtype=torch.int32, device="cuda")
    return a_q, b_q, a_s, b_s, offs


def _with_workspace(lib, _lib, ops, M, N, K, E, schedule):
    a_q, b_q, a_s, b_s, offs = ops
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    wsb = lib.mxgg_grouped_mm_workspace_size(M, N, K, E)
    ws = torch.empty(wsb + 256, dtype=torch.uint8, device="cuda")
    wp = ctypes.c_void_p(ws.data_ptr() + (-ws.data_ptr()) % 256)
    cfg = _lib.gemm_config((0, 0, 0, schedule, 0))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    _lib.check(lib.mxgg_grouped_mm_cfg(_vp(a_q), _vp(b_q), _vp(a_s), _vp(b_s), _vp(offs), M, N, K, E, _vp(out),
                                       _lib.DTYPE_BF16, cfg, wp, wsb, stream), "mxgg_grouped_mm_cfg")
    torch.cuda.synchronize()
    return out


def _noalloc_twice(lib, _lib, ops, M, N, K, E):
    a_q, b_q, a_s, b_s, offs = ops
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    outs = []
    for _ in range(2):
        out = torch.full((M, N), float("nan"), dtype=torch.bfloat16, device="cuda")
        _lib.check(lib.mxgg_grouped_mm_noalloc(_vp(a_q), _vp(b_q), _vp(a_s), _vp(b_s), _vp(offs), M, N, K, E,
                                               _vp(out), _lib.DTYPE_BF16, stream), "mxgg_grouped_mm_noalloc")
        torch.cuda.synchronize()
        outs.append(out)
    return outs


def _oracle_rows(ops, rows):
    """fp32 oracle of the listed output rows (dequantise, then matmul)."""
    a_q, b_q, a_s, b_s, offs = ops
    ends = offs.cpu().numpy()
    groups = np.searchsorted(ends, rows, side="right")
    rt = torch.from_numpy(rows).cuda()
    A_d = O.dequant(u8(a_q[rt]), u8(a_s[rt])).astype(np.float32)
    ref = np.empty((len(rows), b_q.shape[1]), dtype=np.float32)
    for g in np.unique(groups):
        Bd = O.dequant(u8(b_q[g]), u8(b_s[g])).astype(np.float32)
        sel = groups == g
        ref[sel] = A_d[sel] @ Bd.T
    return ref


def test_noalloc_matches_workspace_entry_point():
    from mxgg import _lib
    lib = _lib.load()
    E, M, N, K = 4, 1536, 768, 1024
    ops = _operands(E, M, N, K, 21)
    assert lib.mxgg_grouped_mm_workspace_size(M, N, K, E) <= SCRATCH   # split tail on both sides
    ref = _with_workspace(lib, _lib, ops, M, N, K, E, _lib.SCHED_DEFAULT)
    for out in _noalloc_twice(lib, _lib, ops, M, N, K, E):
        assert torch.equal(out, ref)
    # and both against the oracle
    rows = np.arange(M)
    valid = rows < int(ops[4][-1])
    expect = bf16_round(_oracle_rows(ops, rows[valid]))
    assert O.rel_l2(f32(ref)[valid], expect) <= REL_BF16


def test_noalloc_whole_tiles_when_partials_do_not_fit():
    """Packed scales ~13.6 MB (they fit), split-tail partials ~21 MB more
    (they do not): the call deals whole tiles."""
    from mxgg import _lib
    lib = _lib.load()
    E, M, N, K = 8, 2048, 6144, 8192
    assert lib.mxgg_grouped_mm_workspace_size(M, N, K, E) > SCRATCH
    ops = _operands(E, M, N, K, 22)
    ref = _with_workspace(lib, _lib, ops, M, N, K, E, _lib.SCHED_TILES)
    for out in _noalloc_twice(lib, _lib, ops, M, N, K, E):
        assert torch.equal(out, ref)
    rows = np.sort(np.random.default_rng(0).choice(M, 64, replace=False))
    rows = rows[rows < int(ops[4][-1])]
    got = f32(ref[torch.from_numpy(rows).cuda()])
    assert O.rel_l2(got, bf16_round(_oracle_rows(ops, rows))) <= REL_BF16


def test_noalloc_rejects_oversized_problem():
    from mxgg import _lib
    lib = _lib.load()
    # 64 experts of 8192 x 8192: the packed scales alone exceed the static array
    E, M, N, K = 64, 16640, 8192, 8192
    assert lib.mxgg_grouped_mm_workspace_size(M, N, K, E) > SCRATCH
    dummy = ctypes.c_void_p(256)
    rc = lib.mxgg_grouped_mm_noalloc(dummy, dummy, dummy, dummy, dummy, M, N, K, E, dummy, _lib.DTYPE_BF16,
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 3
    assert "static array" in lib.mxgg_last_error().decode()
