"""Scales laid out once: the blocked scale layout written by the quantiser and
read by the grouped GEMMs in place (``scale_layout="blocked"``).

* The quantiser's blocked output equals a CPU restatement of the layout
  applied to ``to_mx``'s row-major scales, byte for byte (padding zero), and
  its e4m3 data equals ``to_mx``'s.
* Every GEMM pass gives bit-identical outputs (``torch.equal``) from the
  row-major scales (re-laid by the pack launch) and from the blocked scales
  (no pack launch): forward and dgrad over jagged, 16-aligned, empty and
  ragged groups, K off the 128 grid, every tile shape; wgrad and the
  accumulating wgrad.
"""
import numpy as np
import pytest
import torch

from helpers import blocked_scales_ref, gpu_status_clear, offsets, randn_bf16, u8

pytestmark = pytest.mark.gpu


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


def _bounds(ends):
    out, lo = [], 0
    for e in ends:
        out.append((lo, e))
        lo = e
    return out


@pytest.mark.parametrize("M,K,ends", [
    (1024, 512, [100, 100, 612, 1024]),           # ragged, one empty group
    (2048, 160, [256, 1280, 2048]),               # K off the 128 grid (padded k-blocks)
    (512, 1024, [512]),                           # one group
    (768, 256, [16, 48, 768]),                    # groups shorter than a slab
])
def test_quantiser_blocked_groups_layout(U, M, K, ends):
    x = randn_bf16((M, K), seed=M + K)
    offs = torch.tensor(ends, dtype=torch.int32, device="cuda")
    s_blk, q_blk = U.to_mx_grouped_blocked(x, offs)
    s_rm, q_rm = U.to_mx(x)
    assert torch.equal(q_blk.view(torch.uint8), q_rm.view(torch.uint8))
    want = blocked_scales_ref(u8(s_rm), _bounds(ends))
    got = u8(s_blk)
    assert got.shape[0] >= want.shape[0]
    assert np.array_equal(got[:want.shape[0]], want)
    assert not got[want.shape[0]:].any()


def test_quantiser_blocked_experts_layout(U):
    E, N, K = 3, 200, 384            # N off the 128 grid: every expert starts a new slab
    w = randn_bf16((E, N, K), seed=5)
    s_blk, q_blk = U.to_mx_grouped_blocked(w)
    s_rm, q_rm = U.to_mx(w)
    assert torch.equal(q_blk.view(torch.uint8), q_rm.view(torch.uint8))
    want = blocked_scales_ref(u8(s_rm).reshape(E * N, K // 32), [(e * N, (e + 1) * N) for e in range(E)])
    assert np.array_equal(u8(s_blk)[:want.shape[0]], want)


def test_quantiser_dim1_blocked_layout(U):
    M, K = 1024, 320
    x = randn_bf16((M, K), seed=9)
    s_blk, q_blk = U.to_mx_dim1_blocked(x)
    s_rm, q_rm = U.to_mx_dim1(x)
    assert torch.equal(q_blk.view(torch.uint8), q_rm.view(torch.uint8))
    want = blocked_scales_ref(u8(s_rm), [(0, K)])
    assert np.array_equal(u8(s_blk)[:want.shape[0]], want)


def _fwd_pair(K_, U, A, W, offs, tile=None):
    """(row-major result, blocked result) of the same forward call."""
    import mxgg
    a_s, a_q = U.to_mx(A)
    w_s, w_q = U.to_mx(W)
    a_sb, a_qb = U.to_mx_grouped_blocked(A, offs)
    w_sb, w_qb = U.to_mx_grouped_blocked(W)
    if tile is not None:
        mxgg.set_tile_config(*tile)
    try:
        rm = K_.triton_mxfp8_grouped_mm(a_q, w_q, a_s, w_s, offs)
        bl = K_.triton_mxfp8_grouped_mm(a_qb, w_qb, a_sb, w_sb, offs, scale_layout="blocked")
    finally:
        if tile is not None:
            mxgg.set_tile_config(0, 0, 0)
    torch.cuda.synchronize()
    return rm, bl


def _rows(offs):
    return int(offs[-1].item())


@pytest.mark.parametrize("tile", [None, (128, 256, 0), (128, 128, 0), (256, 128, 0)])
@pytest.mark.parametrize("E,M,N,K,mult", [(4, 2048, 1024, 1024, 32), (8, 3072, 512, 2048, 16),
                                          (1, 1000, 384, 160, 8), (6, 1536, 640, 896, 1)])
def test_forward_bit_identical(K_, U, tile, E, M, N, K, mult):
    A = randn_bf16((M, K), seed=E + M)
    W = randn_bf16((E, N, K), seed=E + N, scale=0.05)
    if mult == 1:
        ends = sorted([0, 0, 37, 500, 501, M][:E])   # empty groups, ragged edges
        ends[-1] = M
        offs = torch.tensor(ends, dtype=torch.int32, device="cuda")
    else:
        offs = torch.tensor(offsets(E, M - (M % mult), mult, seed=E), dtype=torch.int32, device="cuda")
    rm, bl = _fwd_pair(K_, U, A, W, offs, tile)
    n = _rows(offs)
    assert torch.equal(rm[:n], bl[:n])


def test_dgrad_bit_identical(K_, U):
    E, M, N, K = 4, 2048, 1536, 1024
    offs = torch.tensor(offsets(E, M, 32, seed=11), dtype=torch.int32, device="cuda")
    GO = randn_bf16((M, N), seed=12)
    W = randn_bf16((E, N, K), seed=13, scale=0.05)
    Wt = W.transpose(-2, -1).contiguous()          # (E, K, N): dgrad's B, contraction N
    rm, bl = _fwd_pair(K_, U, GO, Wt, offs)
    assert torch.equal(rm, bl)


@pytest.mark.parametrize("E,M,N,K", [(4, 2048, 1024, 768), (8, 4096, 512, 1024), (1, 1024, 256, 384)])
def test_wgrad_bit_identical(K_, U, E, M, N, K):
    offs = torch.tensor(offsets(E, M, 32, seed=E), dtype=torch.int32, device="cuda")
    GO = randn_bf16((M, N), seed=21)
    X = randn_bf16((M, K), seed=22)
    go_s, go_q = U.to_mx_dim1(GO)
    x_s, x_q = U.to_mx_dim1(X)
    go_sb, go_qb = U.to_mx_dim1_blocked(GO)
    x_sb, x_qb = U.to_mx_dim1_blocked(X)
    rm = K_.triton_mxfp8_wgrad(go_q, go_s, x_q, x_s, offs)
    bl = K_.triton_mxfp8_wgrad(go_qb, go_sb, x_qb, x_sb, offs, scale_layout="blocked")
    assert torch.equal(rm, bl)
    base = randn_bf16((E, N, K), seed=23).float()
    acc_rm = base.clone()
    acc_bl = base.clone()
    K_.triton_mxfp8_wgrad(go_q, go_s, x_q, x_s, offs, out=acc_rm)
    K_.triton_mxfp8_wgrad(go_qb, go_sb, x_qb, x_sb, offs, out=acc_bl, scale_layout="blocked")
    assert torch.equal(acc_rm, acc_bl)


def test_blocked_call_launches_one_kernel(K_, U):
    """With blocked scales the call is the GEMM launch alone (no pack)."""
    from torch.profiler import ProfilerActivity, profile
    E, M, N, K = 4, 2048, 1024, 1024
    offs = torch.tensor(offsets(E, M, 32, seed=3), dtype=torch.int32, device="cuda")
    a_sb, a_qb = U.to_mx_grouped_blocked(randn_bf16((M, K), seed=1), offs)
    w_sb, w_qb = U.to_mx_grouped_blocked(randn_bf16((E, N, K), seed=2))
    a_s, a_q = U.to_mx(randn_bf16((M, K), seed=1))
    w_s, w_q = U.to_mx(randn_bf16((E, N, K), seed=2))
    K_.triton_mxfp8_grouped_mm(a_qb, w_qb, a_sb, w_sb, offs, scale_layout="blocked")
    torch.cuda.synchronize()

    def kernels_of(fn):
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            fn()
            torch.cuda.synchronize()
        return [e.name for e in prof.events() if e.device_type.name == "CUDA"]

    names_bl = kernels_of(lambda: K_.triton_mxfp8_grouped_mm(a_qb, w_qb, a_sb, w_sb, offs, scale_layout="blocked"))
    names_rm = kernels_of(lambda: K_.triton_mxfp8_grouped_mm(a_q, w_q, a_s, w_s, offs))
    mx_bl = [n for n in names_bl if "mxgg" in n]
    mx_rm = [n for n in names_rm if "mxgg" in n]
    assert any("grouped_gemm" in n for n in mx_bl) and not any("pack_scales" in n for n in mx_bl), mx_bl
    assert any("pack_scales" in n for n in mx_rm), mx_rm
