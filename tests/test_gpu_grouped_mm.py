"""Forward / dgrad grouped GEMM on the GPU against the oracle.

Tolerances (floating point, from the path's spec): rel-L2 <= 1e-3 against the
dequantise-then-fp32 emulation for bf16 outputs (both sides rounded to bf16),
<= 1e-5 for fp32 outputs, and SQNR >= 27 dB against a bf16 grouped matmul of
the unquantised inputs (the reference's own gate, test_correctness.py:26).
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import O, bf16_round, f32, gpu_status_clear, offsets, u8

pytestmark = pytest.mark.gpu

REL_BF16 = 1e-3
REL_F32 = 1e-5


@pytest.fixture(scope="module")
def K_():
    import kernels
    assert kernels._mxfp8_available, "sm_100a kernels must be available on the GPU box"
    return kernels


@pytest.fixture(scope="module")
def U():
    import utils
    return utils


@pytest.fixture(autouse=True)
def _status():
    gpu_status_clear()
    yield
    assert gpu_status_clear() == 0, "a device-side wait timed out"


def _make(E, M, N, K, offs, seed=0, bscale=1.0, dtype=torch.bfloat16):
    import utils
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(dtype).cuda()
    B = (torch.randn(E, N, K, generator=g) * bscale).to(dtype).cuda()
    a_s, a_q = utils.to_mx(A)
    b_s, b_q = utils.to_mx(B)
    return A, B, a_s, a_q, b_s, b_q, torch.tensor(offs, dtype=torch.int32, device="cuda")


def _oracle(a_q, a_s, b_q, b_s, offs):
    return O.grouped_mm(u8(a_q), u8(a_s), u8(b_q), u8(b_s), offs.cpu().numpy(), acc=np.float32)


def _check(out, ref, out_dtype):
    valid = ~np.isnan(ref)
    got = f32(out)[valid]
    if out_dtype == torch.float32:
        err = O.rel_l2(got, ref[valid])
        assert err <= REL_F32, err
    else:
        err = O.rel_l2(got, bf16_round(ref)[valid])
        assert err <= REL_BF16, err
    return err


def test_golden_config1(K_, golden):
    dev = lambda k, dt=torch.uint8: torch.from_numpy(golden[k]).cuda().view(dt)  # noqa: E731
    a_q, a_s = dev("fwd1_a_q", torch.float8_e4m3fn), dev("fwd1_a_s")
    b_q, b_s = dev("fwd1_b_q", torch.float8_e4m3fn), dev("fwd1_b_s")
    offs = torch.from_numpy(golden["fwd1_offs"]).cuda()
    ref = golden["fwd1_out_f32"]
    for out_dtype in (torch.bfloat16, torch.float32):
        out = K_.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, offs, out_dtype=out_dtype)
        torch.cuda.synchronize()
        _check(out, ref, out_dtype)
    out = K_.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, offs)
    hp = O.bf16_bits_to_f32(golden["fwd1_hp_bf16"])
    assert O.compute_error(hp, f32(out)) >= 27.0


@pytest.mark.parametrize("E,M,N,K", [(1, 1024, 1024, 1024), (8, 1024, 4096, 2048),
                                     (4, 1024, 2048, 2048), (8, 2048, 5120, 2048)])
def test_reference_shapes_sqnr(K_, U, E, M, N, K):
    """The reference's own correctness shapes (test_correctness.py:70-73)."""
    torch.manual_seed(0)
    A = torch.randn((M, K), dtype=torch.bfloat16, device="cuda")
    B = torch.randn((E, N, K), dtype=torch.bfloat16, device="cuda")
    a_s, a_q = U.to_mx(A)
    b_s, b_q = U.to_mx(B)
    offs = torch.tensor(offsets(E, M, 32, seed=E + M), dtype=torch.int32, device="cuda")
    out = K_.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, offs)
    ref_hp = torch._grouped_mm(A, B.transpose(-2, -1), offs=offs, out_dtype=torch.bfloat16)
    sqnr = O.compute_error(f32(ref_hp), f32(out))
    assert sqnr >= 27.0, sqnr
    _check(out, _oracle(a_q, a_s, b_q, b_s, offs), torch.bfloat16)


@pytest.mark.parametrize("tile_m,tile_n", [(128, 128), (128, 256), (256, 128), (256, 256)])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_tile_configs_and_dtypes(K_, tile_m, tile_n, out_dtype):
    import mxgg
    E, M, N, K = 3, 700, 512, 384
    offs = [96, 96 + 352, 700]
    _, _, a_s, a_q, b_s, b_q, o = _make(E, M, N, K, offs, seed=3)
    mxgg.set_tile_config(tile_m, tile_n, 0)
    try:
        out = K_.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, o, out_dtype=out_dtype)
        torch.cuda.synchronize()
    finally:
        mxgg.set_tile_config(0, 0, 0)
    ref = _oracle(a_q, a_s, b_q, b_s, o)
    if out_dtype == torch.float16:
        valid = ~np.isnan(ref)
        assert O.rel_l2(f32(out)[valid], ref[valid]) <= 1e-3
    else:
        _check(out, ref, out_dtype)


@pytest.mark.parametrize("case", ["empty_groups", "single_group", "unaligned16", "ragged", "tail_rows",
                                  "k_tail", "n_tail", "n_odd", "many_groups"])
def test_edge_cases(K_, case):
    E, M, N, K = 4, 1000, 256, 512
    if case == "empty_groups":
        E, M = 5, 640
        offs = [0, 256, 256, 640, 640]
    elif case == "single_group":
        E, M = 1, 999
        offs = [999]
    elif case == "unaligned16":
        E, M = 4, 1024
        offs = [16, 400, 656, 1024]
    elif case == "ragged":
        E, M = 4, 1000
        offs = [1, 130, 131, 1000]
    elif case == "tail_rows":
        E, M = 3, 1024
        offs = [128, 320, 800]     # rows 800.. are not written
    elif case == "k_tail":
        E, M, K = 2, 512, 544      # K % 128 != 0: partial last stage + byte-gather scale path
        offs = [200, 512]
    elif case == "n_tail":
        E, M, N = 2, 512, 200      # N % tile != 0, still 16-byte rows
        offs = [300, 512]
    elif case == "n_odd":
        E, M, N = 2, 384, 100      # rows not 16-byte aligned: predicated stores
        offs = [64, 384]
    elif case == "many_groups":
        E, M, N, K = 64, 4096, 256, 256
        offs = list(offsets(64, 4096, 32, seed=5))
    _, _, a_s, a_q, b_s, b_q, o = _make(E, M, N, K, offs, seed=11)
    # fill the output with a sentinel through the C ABI so unwritten rows are visible
    out = torch.full((M, N), 7.0, dtype=torch.bfloat16, device="cuda")
    from mxgg import _lib
    lib = _lib.load()
    wsb = lib.mxgg_grouped_mm_workspace_size(M, N, K, E)
    ws = torch.empty(wsb + 1024, dtype=torch.uint8, device="cuda")
    wp = ws.data_ptr() + (-ws.data_ptr()) % 1024
    rc = lib.mxgg_grouped_mm(ctypes.c_void_p(a_q.data_ptr()), ctypes.c_void_p(b_q.data_ptr()),
                             ctypes.c_void_p(a_s.data_ptr()), ctypes.c_void_p(b_s.data_ptr()),
                             ctypes.c_void_p(o.data_ptr()), M, N, K, E, ctypes.c_void_p(out.data_ptr()),
                             _lib.DTYPE_BF16, ctypes.c_void_p(wp), wsb,
                             ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "mxgg_grouped_mm")
    torch.cuda.synchronize()
    ref = _oracle(a_q, a_s, b_q, b_s, o)
    _check(out, ref, torch.bfloat16)
    tail = int(max(offs))
    if tail < M:
        assert torch.all(out[tail:] == 7.0), "rows past the last group end must stay untouched"


def test_full_size_sampled_rows(K_, U):
    """A full Llama4 sweep shape (E=8, N=K=8192) checked on sampled rows."""
    E, M, N, K = 8, 16640, 8192, 8192
    offs = O.llama4_offsets(123)[35]
    torch.manual_seed(123)
    A = torch.randn(M, K, dtype=torch.bfloat16, device="cuda")
    B = torch.randn(E, N, K, dtype=torch.bfloat16, device="cuda")
    a_s, a_q = U.to_mx(A)
    b_s, b_q = U.to_mx(B)
    del A, B
    o = torch.tensor(offs, dtype=torch.int32, device="cuda")
    out = K_.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, o)
    torch.cuda.synchronize()
    rng = np.random.default_rng(0)
    rows = np.sort(rng.choice(M, 48, replace=False))
    groups = np.searchsorted(np.asarray(offs), rows, side="right")
    rt = torch.from_numpy(rows).cuda()
    A_d = O.dequant(u8(a_q[rt]), u8(a_s[rt])).astype(np.float32)
    got = f32(out[rt])
    ref = np.empty_like(got)
    for g in np.unique(groups):
        Bd = O.dequant(u8(b_q[g]), u8(b_s[g])).astype(np.float32)
        sel = groups == g
        ref[sel] = A_d[sel] @ Bd.T
    assert O.rel_l2(got, bf16_round(ref)) <= REL_BF16


@pytest.mark.parametrize("E,N,K,passname", [(8, 5120, 2048, "fwd"), (4, 2048, 8192, "fwd"), (8, 2048, 5120, "dgrad")])
def test_full_size_mult16_sampled_rows(K_, U, E, N, K, passname):
    """BASELINE config 2/3 group sizes: multiples of 16 (so group edges fall
    mid 32-row block) at the sweep's full M, checked on sampled rows that
    include every group's first and last row."""
    import random
    M = 16640
    random.seed(1600 + E)
    offs = U.generate_jagged_offs(E, M, multiple_of=16, device="cpu").tolist()
    assert any(o % 32 for o in offs[:-1]), "the draw must put a group edge off the 32-row grid"
    torch.manual_seed(16)
    if passname == "fwd":
        A = torch.randn(M, K, dtype=torch.bfloat16, device="cuda")
        B = torch.randn(E, N, K, dtype=torch.bfloat16, device="cuda")
        a_s, a_q = U.to_mx(A)
        b_s, b_q = U.to_mx(B)
    else:
        # dgrad: grad_out (M, N) and W^T (E, K, N), both quantised along N
        A = torch.randn(M, N, dtype=torch.bfloat16, device="cuda")
        B = torch.randn(E, N, K, dtype=torch.bfloat16, device="cuda")
        a_s, a_q = U.to_mx(A)
        wt = [U.to_mx_dim1(B[e]) for e in range(E)]
        b_s = torch.stack([s_ for s_, _ in wt])
        b_q = torch.stack([q for _, q in wt])
    del A, B
    o = torch.tensor(offs, dtype=torch.int32, device="cuda")
    out = K_.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, o)
    torch.cuda.synchronize()
    starts = [0] + offs[:-1]
    edges = sorted({r for a, b in zip(starts, offs) if b > a for r in (a, b - 1)})
    rng = np.random.default_rng(1)
    rows = np.array(sorted(set(edges) | set(rng.choice(M, 32, replace=False).tolist())))
    groups = np.searchsorted(np.asarray(offs), rows, side="right")
    rt = torch.from_numpy(rows).cuda()
    A_d = O.dequant(u8(a_q[rt]), u8(a_s[rt])).astype(np.float32)
    got = f32(out[rt])
    ref = np.empty_like(got)
    for g in np.unique(groups):
        Bd = O.dequant(u8(b_q[g]), u8(b_s[g])).astype(np.float32)
        sel = groups == g
        ref[sel] = A_d[sel] @ Bd.T
    assert O.rel_l2(got, bf16_round(ref)) <= REL_BF16


def test_dgrad_pass(K_, U):
    """dgrad = the same op with grad_out (M, N) and W^T (E, K, N), both
    quantised along N (the contraction)."""
    E, M, N, K = 4, 1536, 640, 384
    offs = offsets(E, M, 32, seed=9)
    g = torch.Generator().manual_seed(9)
    go = torch.randn(M, N, generator=g).to(torch.bfloat16).cuda()
    W = torch.randn(E, N, K, generator=g).to(torch.bfloat16).cuda()
    go_s, go_q = U.to_mx(go)
    wt_s, wt_q = U.to_mx(W.transpose(-2, -1).contiguous())
    o = torch.tensor(offs, dtype=torch.int32, device="cuda")
    dx = K_.triton_mxfp8_grouped_mm(go_q, wt_q, go_s, wt_s, o)
    assert dx.shape == (M, K)
    _check(dx, _oracle(go_q, go_s, wt_q, wt_s, o), torch.bfloat16)
    hp = torch._grouped_mm(go, W, offs=o, out_dtype=torch.bfloat16)
    assert O.compute_error(f32(hp), f32(dx)) >= 27.0


def test_tile_map_matches_reference_layout(K_):
    import mxgg
    for offs, M, bm in [([100, 100, 356, 1000], 1000, 128), (list(offsets(8, 16640, 32, 3)), 16640, 256),
                        ([0, 0, 64], 64, 64)]:
        o = torch.tensor(offs, dtype=torch.int32, device="cuda")
        got = mxgg.build_tile_map(o, M, bm).cpu().numpy()
        hist, raw, pad, pmap = O.build_tile_map(offs, M, bm)
        E = len(offs)
        np.testing.assert_array_equal(got[:E], hist)
        np.testing.assert_array_equal(got[E:2 * E], raw)
        assert got[2 * E] == pad
        np.testing.assert_array_equal(got[2 * E + 1:], pmap)


@pytest.mark.parametrize("sched,split_max", [(1, 0), (2, 0), (2, 64)])
@pytest.mark.parametrize("tile_m", [128, 256])
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("E,M,N,K,offs", [
    # fewer tiles than pairs: every tile split along K
    (1, 2048, 256, 4096, [2048]),
    # a full round of tiles, then a partial one that is split
    (2, 2048, 2560, 1024, [1000, 2048]),
    # ragged groups, odd N (predicated stores), an empty group
    (4, 1500, 200, 2048, [300, 300, 1100, 1500]),
])
def test_split_tail_schedule(K_, sched, split_max, tile_m, out_dtype, E, M, N, K, offs):
    """Whole-tile and split-tail schedules against the oracle."""
    import mxgg
    _, _, a_s, a_q, b_s, b_q, o = _make(E, M, N, K, offs, seed=E + K)
    mxgg.set_schedule(sched, split_max)
    mxgg.set_tile_config(tile_m, 0, 0)
    try:
        out = K_.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, o, out_dtype=out_dtype)
        torch.cuda.synchronize()
    finally:
        mxgg.set_schedule(0, 0)
        mxgg.set_tile_config(0, 0, 0)
    _check(out, _oracle(a_q, a_s, b_q, b_s, o), out_dtype)


def test_split_tail_deterministic(K_):
    import mxgg
    E, M, N, K = 1, 2048, 512, 8192
    _, _, a_s, a_q, b_s, b_q, o = _make(E, M, N, K, [M], seed=4)
    mxgg.set_schedule(2, 64)
    try:
        outs = [K_.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, o, out_dtype=torch.float32) for _ in range(4)]
        torch.cuda.synchronize()
    finally:
        mxgg.set_schedule(0, 0)
    for x in outs[1:]:
        assert torch.equal(x, outs[0])
