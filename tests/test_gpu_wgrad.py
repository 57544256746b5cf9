"""Weight-gradient grouped GEMM on the GPU against the oracle.

rel-L2 <= 1e-3 for bf16 outputs (compared after rounding the oracle to bf16),
<= 1e-5 for fp32 outputs; empty groups must be exact zeros.
"""
import numpy as np
import pytest
import torch

from helpers import O, bf16_round, f32, gpu_status_clear, offsets, u8
from mxgg import _lib

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def K_():
    import kernels
    assert kernels._mxfp8_available
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


def _inputs(M, N, K, seed):
    import utils
    g = torch.Generator().manual_seed(seed)
    go = torch.randn(M, N, generator=g).to(torch.bfloat16).cuda()
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    go_s, go_q = utils.to_mx_dim1(go)      # (N, M/32), (N, M)
    ia_s, ia_q = utils.to_mx_dim1(x)       # (K, M/32), (K, M)
    return go, x, go_s, go_q, ia_s, ia_q


def _oracle(go_q, go_s, ia_q, ia_s, offs):
    return O.wgrad(u8(go_q), u8(go_s), u8(ia_q), u8(ia_s), np.asarray(offs), acc=np.float32)


def _check(out, ref, out_dtype):
    if out_dtype == torch.float32:
        err = O.rel_l2(f32(out), ref)
        assert err <= 1e-5, err
    else:
        err = O.rel_l2(f32(out), bf16_round(ref))
        assert err <= 1e-3, err


def test_golden_small(K_, golden):
    dev = lambda k, dt=torch.uint8: torch.from_numpy(golden[k]).cuda().view(dt)  # noqa: E731
    out = K_.triton_mxfp8_wgrad(dev("wg_go_q", torch.float8_e4m3fn), dev("wg_go_s"),
                                dev("wg_ia_q", torch.float8_e4m3fn), dev("wg_ia_s"),
                                torch.from_numpy(golden["wg_offs"]).cuda(), out_dtype=torch.float32)
    torch.cuda.synchronize()
    _check(out, golden["wg_out_f32"], torch.float32)


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("E,M,N,K", [(1, 1024, 256, 512), (4, 2048, 384, 256), (8, 4096, 256, 768)])
def test_random_vs_oracle(K_, out_dtype, E, M, N, K):
    offs = offsets(E, M, 32, seed=E * 7 + K)
    _, _, go_s, go_q, ia_s, ia_q = _inputs(M, N, K, seed=E)
    o = torch.tensor(offs, dtype=torch.int32, device="cuda")
    out = K_.triton_mxfp8_wgrad(go_q, go_s, ia_q, ia_s, o, out_dtype=out_dtype)
    torch.cuda.synchronize()
    _check(out, _oracle(go_q, go_s, ia_q, ia_s, offs), out_dtype)


def test_empty_and_unaligned_groups(K_):
    # groups that start/end off the 128-token stage grid, and empty groups
    E, M, N, K = 6, 1024, 256, 256
    offs = [0, 32, 32, 480, 992, 1024]
    _, _, go_s, go_q, ia_s, ia_q = _inputs(M, N, K, seed=5)
    o = torch.tensor(offs, dtype=torch.int32, device="cuda")
    out = K_.triton_mxfp8_wgrad(go_q, go_s, ia_q, ia_s, o, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ref = _oracle(go_q, go_s, ia_q, ia_s, offs)
    _check(out, ref, torch.float32)
    assert torch.count_nonzero(out[0]) == 0 and torch.count_nonzero(out[2]) == 0


def test_tokens_not_multiple_of_128(K_):
    # M % 128 != 0 -> scale rows are not 4-byte aligned: byte-gather path
    E, M, N, K = 3, 544, 128, 256
    offs = [96, 320, 544]
    _, _, go_s, go_q, ia_s, ia_q = _inputs(M, N, K, seed=8)
    o = torch.tensor(offs, dtype=torch.int32, device="cuda")
    out = K_.triton_mxfp8_wgrad(go_q, go_s, ia_q, ia_s, o, out_dtype=torch.float32)
    torch.cuda.synchronize()
    _check(out, _oracle(go_q, go_s, ia_q, ia_s, offs), torch.float32)


def test_matches_hp_sqnr(K_):
    E, M, N, K = 4, 2048, 512, 512
    offs = offsets(E, M, 32, seed=2)
    go, x, go_s, go_q, ia_s, ia_q = _inputs(M, N, K, seed=2)
    o = torch.tensor(offs, dtype=torch.int32, device="cuda")
    out = K_.triton_mxfp8_wgrad(go_q, go_s, ia_q, ia_s, o)
    ref = torch.zeros(E, N, K, device="cuda")
    prev = 0
    for g, e in enumerate(offs):
        ref[g] = go[prev:e].float().t() @ x[prev:e].float()
        prev = e
    assert O.compute_error(f32(ref), f32(out)) >= 27.0


def test_full_size_sampled(K_, U):
    """Full Llama4 sweep shape E=8, N=K=8192 checked on sampled output rows."""
    E, M, N, K = 8, 16640, 8192, 8192
    offs = O.llama4_offsets(123)[35]
    g = torch.Generator(device="cuda").manual_seed(0)
    go = torch.randn(M, N, device="cuda", dtype=torch.bfloat16, generator=g)
    go_s, go_q = U.to_mx_dim1(go)
    del go
    x = torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g)
    ia_s, ia_q = U.to_mx_dim1(x)
    del x
    o = torch.tensor(offs, dtype=torch.int32, device="cuda")
    out = K_.triton_mxfp8_wgrad(go_q, go_s, ia_q, ia_s, o)
    torch.cuda.synchronize()
    rng = np.random.default_rng(1)
    rows = np.sort(rng.choice(N, 16, replace=False))
    cols = np.sort(rng.choice(K, 64, replace=False))
    rt, ct = torch.from_numpy(rows).cuda(), torch.from_numpy(cols).cuda()
    GOd = O.dequant(u8(go_q[rt]), u8(go_s[rt])).astype(np.float32)       # (16, M)
    IAd = O.dequant(u8(ia_q[ct]), u8(ia_s[ct])).astype(np.float32)       # (64, M)
    got_all = f32(out[:, rt][:, :, ct])
    prev = 0
    for gi, e in enumerate(offs):
        ref = GOd[:, prev:e] @ IAd[:, prev:e].T
        assert O.rel_l2(got_all[gi], bf16_round(ref)) <= 1e-3
        prev = e


@pytest.fixture
def schedule():
    """Set the GEMM schedule for one test and restore the defaults after it."""
    def set_(s, split_max=0):
        _lib.set_schedule(s, split_max)
    yield set_
    _lib.set_schedule(_lib.SCHED_DEFAULT, 0)
    _lib.set_tile_config(0, 0, 0)


@pytest.mark.parametrize("sched,split_max", [(_lib.SCHED_TILES, 0), (_lib.SCHED_SPLIT_TAIL, 0),
                                             (_lib.SCHED_SPLIT_TAIL, 64)])
@pytest.mark.parametrize("tile_m", [128, 256])
@pytest.mark.parametrize("E,M,N,K,offs", [
    # one tile: split over as many pairs as it has stages (split_max 64)
    (1, 8192, 256, 256, [8192]),
    # a few tiles, many stages: every tile split across several pairs
    (2, 16384, 256, 512, [9600, 16384]),
    # jagged groups (empty, sub-stage, off-grid); the tail holds empty-group tiles
    (5, 2048, 384, 256, [0, 32, 480, 480, 2048]),
    # many tiles: a full round and a partial one
    (8, 4096, 1024, 2560, None),
])
def test_schedules_vs_oracle(K_, schedule, sched, split_max, tile_m, E, M, N, K, offs):
    schedule(sched, split_max)
    _lib.set_tile_config(tile_m, 0, 0)
    if offs is None:
        offs = offsets(E, M, 32, seed=11)
    _, _, go_s, go_q, ia_s, ia_q = _inputs(M, N, K, seed=E + 3)
    o = torch.tensor(offs, dtype=torch.int32, device="cuda")
    out = K_.triton_mxfp8_wgrad(go_q, go_s, ia_q, ia_s, o, out_dtype=torch.float32)
    torch.cuda.synchronize()
    ref = _oracle(go_q, go_s, ia_q, ia_s, offs)
    _check(out, ref, torch.float32)
    prev = 0
    for g, e in enumerate(offs):
        if e == prev:
            assert torch.count_nonzero(out[g]) == 0
        prev = e


def test_split_tail_deterministic(K_, schedule):
    """Partials are summed in a fixed order: repeated calls are bit-identical."""
    schedule(_lib.SCHED_SPLIT_TAIL, 64)
    E, M, N, K = 3, 12288, 512, 512
    offs = [4000, 4000, 12288]
    _, _, go_s, go_q, ia_s, ia_q = _inputs(M, N, K, seed=9)
    o = torch.tensor(offs, dtype=torch.int32, device="cuda")
    outs = [K_.triton_mxfp8_wgrad(go_q, go_s, ia_q, ia_s, o, out_dtype=torch.float32) for _ in range(4)]
    torch.cuda.synchronize()
    for x in outs[1:]:
        assert torch.equal(x, outs[0])


@pytest.mark.parametrize("sched", [_lib.SCHED_TILES, _lib.SCHED_SPLIT_TAIL])
@pytest.mark.parametrize("N", [384, 360])       # 360: warps cut by the tile edge read-add-write instead of TMA reduce
def test_wgrad_accumulate_into_fp32(K_, schedule, sched, N):
    """out += wgrad, one fp32 add per element: bit-exact against the plain
    fp32 result added in torch (same schedule, so the same products)."""
    schedule(sched, 64)
    E, M, K = 3, 4096, 512
    offs = [1024, 1024, 4096]
    _, _, go_s, go_q, ia_s, ia_q = _inputs(M, N, K, seed=21)
    o = torch.tensor(offs, dtype=torch.int32, device="cuda")
    fresh = K_.triton_mxfp8_wgrad(go_q, go_s, ia_q, ia_s, o, out_dtype=torch.float32)
    base = torch.randn(E, N, K, generator=torch.Generator().manual_seed(3)).cuda()
    want = base + fresh
    got = K_.triton_mxfp8_wgrad(go_q, go_s, ia_q, ia_s, o, out=base)
    torch.cuda.synchronize()
    assert got is base
    assert torch.equal(got, want)
