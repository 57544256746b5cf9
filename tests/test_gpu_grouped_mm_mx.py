"""Forward GEMM with to_mx of its output fused into the epilogue, on the GPU.

The fused outputs must be bit for bit what ``to_mx`` (rows) and
``to_mx_dim1`` (the transpose, quantised along tokens) give for the GEMM's own
bf16 / f16 output (integer and byte work: exact).  Checked twice: against the
separate GPU calls (``triton_mxfp8_grouped_mm`` then ``utils.to_mx`` /
``utils.to_mx_dim1``) and against the oracle's FLOOR-mode ``to_mx`` (pinned to
the reference's utils.py:67-105) applied to that output on the CPU.  Rows at
or past the last group end are not written and are not compared.
"""
import numpy as np
import pytest
import torch

from helpers import O, gpu_status_clear, offsets, u8

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status():
    gpu_status_clear()
    yield
    assert gpu_status_clear() == 0, "a device-side wait timed out"


def _roll(q, k):
    """Rows of an e4m3 tensor rotated by k (torch has no fp8 roll)."""
    return q.view(torch.uint8).roll(k, 0).view(q.dtype)


def _make(E, M, N, K, offs, seed=0, fp4=False):
    import utils
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    B = (torch.randn(E, N, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
    a_s, a_q = utils.to_mx(A)
    b_s, b_q = utils.to_mx(B, elem_dtype=torch.float4_e2m1fn_x2) if fp4 else utils.to_mx(B)
    return a_q, b_q, a_s, b_s, torch.tensor(offs, dtype=torch.int32, device="cuda")


def _check(args, out_dtype=torch.bfloat16):
    import kernels
    import utils
    offs = args[-1]
    rows = int(offs[-1].item()) if offs.numel() else 0
    # a first call on other rows, whose freed buffers the calls below may be
    # handed: a row they failed to write then holds a wrong value
    kernels.mxfp8_grouped_mm_to_mx(_roll(args[0], 1), *args[1:], out_dtype=out_dtype, return_output=True)
    out = kernels.triton_mxfp8_grouped_mm(*args, out_dtype=out_dtype)
    s, q = kernels.mxfp8_grouped_mm_to_mx(*args, out_dtype=out_dtype)
    s2, q2, out2 = kernels.mxfp8_grouped_mm_to_mx(*args, out_dtype=out_dtype, return_output=True)
    torch.cuda.synchronize()
    M, N = out.shape
    assert s.shape == (M, N // 32) and s.dtype == torch.uint8
    assert q.shape == (M, N) and q.dtype == torch.float8_e4m3fn
    out, out2 = out[:rows], out2[:rows]
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))
    rs, rq = utils.to_mx(out)
    assert np.array_equal(u8(s[:rows]), u8(rs))
    assert np.array_equal(u8(q[:rows]), u8(rq))
    assert np.array_equal(u8(s2[:rows]), u8(rs)) and np.array_equal(u8(q2[:rows]), u8(rq))
    os_, oq = O.to_mx(out.float().cpu().numpy())
    assert np.array_equal(u8(s[:rows]), os_)
    assert np.array_equal(u8(q[:rows]), oq)
    if M % 32 == 0 and all(int(o) % 32 == 0 for o in offs.tolist()):
        s3, q3, st, qt = kernels.mxfp8_grouped_mm_to_mx(*args, out_dtype=out_dtype, dim1=True)
        torch.cuda.synchronize()
        assert st.shape == (N, M // 32) and qt.shape == (N, M)
        assert np.array_equal(u8(s3[:rows]), u8(rs)) and np.array_equal(u8(q3[:rows]), u8(rq))
        ts, tq = utils.to_mx_dim1(out)
        assert np.array_equal(u8(st[:, :rows // 32]), u8(ts))
        assert np.array_equal(u8(qt[:, :rows]), u8(tq))
        ots, otq = O.to_mx(np.ascontiguousarray(out.float().cpu().numpy().T))
        assert np.array_equal(u8(st[:, :rows // 32]), ots)
        assert np.array_equal(u8(qt[:, :rows]), otq)


@pytest.mark.parametrize("E,M,N,K", [(4, 1024, 256, 512), (1, 640, 2048, 256), (8, 2080, 512, 1024),
                                     (3, 416, 96, 128)])
def test_fused_to_mx_bit_exact(E, M, N, K):
    offs = offsets(E, M, 32, seed=E + N)
    _check(_make(E, M, N, K, offs, seed=1))


def test_fused_to_mx_ragged_and_empty_groups():
    # groups of 0, 16 and 48 rows, a tail past the last group end
    offs = [0, 16, 16, 64, 300, 300]
    _check(_make(6, 400, 256, 256, offs, seed=2))


def test_fused_to_mx_f16_output():
    offs = offsets(2, 512, 32, seed=3)
    _check(_make(2, 512, 256, 256, offs, seed=3), out_dtype=torch.float16)


def test_fused_to_mx_e2m1_weights():
    offs = offsets(4, 768, 32, seed=4)
    _check(_make(4, 768, 512, 512, offs, seed=4, fp4=True))


@pytest.mark.parametrize("schedule", ["tiles", "split"])
def test_fused_to_mx_schedules(schedule):
    """Split-tail tiles (reduced in the last pair's epilogue) quantise too."""
    import mxgg
    mxgg.set_schedule(mxgg._lib.SCHED_TILES if schedule == "tiles" else mxgg._lib.SCHED_SPLIT_TAIL,
                      2 if schedule == "split" else 0)
    try:
        offs = offsets(2, 2048, 32, seed=5)
        _check(_make(2, 2048, 2048, 4096, offs, seed=5))
    finally:
        mxgg.set_schedule(mxgg._lib.SCHED_DEFAULT, 0)


def test_fused_to_mx_empty_contraction_and_errors():
    import kernels
    a_q, b_q, a_s, b_s, offs = _make(2, 64, 64, 32, [32, 64], seed=6)
    z = torch.empty(64, 0, dtype=torch.float8_e4m3fn, device="cuda")
    zs = torch.empty(64, 0, dtype=torch.uint8, device="cuda")
    zb = torch.empty(2, 64, 0, dtype=torch.float8_e4m3fn, device="cuda")
    zbs = torch.empty(2, 64, 0, dtype=torch.uint8, device="cuda")
    s, q = kernels.mxfp8_grouped_mm_to_mx(z, zb, zs, zbs, offs)
    torch.cuda.synchronize()
    assert not u8(s).any() and not u8(q).any()
    a_q, b_q, a_s, b_s, offs = _make(2, 64, 48, 64, [32, 64], seed=6)
    with pytest.raises(ValueError):
        kernels.mxfp8_grouped_mm_to_mx(a_q, b_q, a_s, b_s, offs)
    with pytest.raises(TypeError):
        kernels.mxfp8_grouped_mm_to_mx(a_q, b_q, a_s, b_s, offs, out_dtype=torch.float32)


def test_fused_to_mx_segments_sharing_experts():
    """Segments that reuse experts (the expert-parallel receive layout): the
    fused output equals to_mx of mxgg::grouped_mm_segments' output."""
    import mxgg
    import utils
    a_q, b_q, a_s, b_s, _ = _make(3, 640, 512, 256, [640], seed=7)
    seg_offs = torch.tensor([64, 192, 192, 352, 640], dtype=torch.int32, device="cuda")   # on the 32-row grid
    seg_e = torch.tensor([0, 2, 1, 0, 1], dtype=torch.int32, device="cuda")
    mxgg.grouped_mm_mx_op(_roll(a_q, 3), b_q, a_s, b_s, seg_offs, seg_e, torch.bfloat16, True, True, True)
    out = mxgg.grouped_mm_segments_op(a_q, b_q, a_s, b_s, seg_offs, seg_e, torch.bfloat16)
    s, q, st, qt, out2 = mxgg.grouped_mm_mx_op(a_q, b_q, a_s, b_s, seg_offs, seg_e, torch.bfloat16, True, True, True)
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), out2.view(torch.int16))
    rs, rq = utils.to_mx(out)
    assert np.array_equal(u8(s), u8(rs)) and np.array_equal(u8(q), u8(rq))
    ts, tq = utils.to_mx_dim1(out)
    assert np.array_equal(u8(st), u8(ts)) and np.array_equal(u8(qt), u8(tq))


def test_fused_dim1_only_and_off_grid_groups():
    """dim1 without the row-wise output; a group starting off the 32-row grid
    raises device status bit 256 (its blocks are skipped), the row-wise
    output stays exact."""
    import mxgg
    import utils
    a_q, b_q, a_s, b_s, offs = _make(2, 256, 256, 256, [128, 256], seed=8)
    _, _, st, qt, out = mxgg.grouped_mm_mx_op(a_q, b_q, a_s, b_s, offs, None, torch.bfloat16, True, False, True)
    torch.cuda.synchronize()
    ts, tq = utils.to_mx_dim1(out)
    assert np.array_equal(u8(st), u8(ts)) and np.array_equal(u8(qt), u8(tq))
    assert mxgg.device_status(clear=True) == 0
    offs = torch.tensor([48, 256], dtype=torch.int32, device="cuda")
    s, q, _, _, out = mxgg.grouped_mm_mx_op(a_q, b_q, a_s, b_s, offs, None, torch.bfloat16, True, True, True)
    torch.cuda.synchronize()
    assert mxgg.device_status(clear=True) & 256
    rs, rq = utils.to_mx(out)
    assert np.array_equal(u8(s), u8(rs)) and np.array_equal(u8(q), u8(rq))
