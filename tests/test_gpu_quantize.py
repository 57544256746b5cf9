"""to_mx on the GPU: bit-exact against the reference's own vectors and the
oracle (integer / byte work: no tolerance)."""
import numpy as np
import pytest
import torch

from helpers import O, as_oracle_input, u8

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def U():
    import utils
    return utils


def _bf16_from_bits(bits):
    return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).cuda()


def _f32_from_bits(bits):
    return torch.from_numpy(bits.view(np.int32)).view(torch.float32).cuda()


def test_golden_bf16(U, golden):
    s, q = U.to_mx(_bf16_from_bits(golden["tomx_bf16_x"]))
    np.testing.assert_array_equal(u8(s), golden["tomx_bf16_s"])
    np.testing.assert_array_equal(u8(q), golden["tomx_bf16_q"])


def test_golden_edge_blocks(U, golden):
    s, q = U.to_mx(_f32_from_bits(golden["tomx_edge_x"]))
    np.testing.assert_array_equal(u8(s), golden["tomx_edge_s"])
    np.testing.assert_array_equal(u8(q), golden["tomx_edge_q"])


def test_golden_3d_fp32(U, golden):
    x = _f32_from_bits(golden["tomx_f32_x"])
    s, q = U.to_mx(x)
    assert s.shape == (3, 17, 3) and q.shape == (3, 17, 96)
    np.testing.assert_array_equal(u8(s), golden["tomx_f32_s"])
    np.testing.assert_array_equal(u8(q), golden["tomx_f32_q"])


def test_golden_config1_operands(U, golden):
    a = _bf16_from_bits(golden["fwd1_a_bits"])
    s, q = U.to_mx(a)
    np.testing.assert_array_equal(u8(s), golden["fwd1_a_s"])
    np.testing.assert_array_equal(u8(q), golden["fwd1_a_q"])
    b = _bf16_from_bits(golden["fwd1_b_bits"])
    s, q = U.to_mx(b)
    np.testing.assert_array_equal(u8(s), golden["fwd1_b_s"])
    np.testing.assert_array_equal(u8(q), golden["fwd1_b_q"])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("shape", [(1, 32), (7, 96), (333, 512), (1024, 2048)])
def test_random_vs_oracle(U, dtype, shape):
    g = torch.Generator().manual_seed(hash((str(dtype), shape)) % 1000)
    x = torch.randn(shape, generator=g) * torch.exp2(torch.randint(-20, 20, (shape[0], 1), generator=g).float())
    x = x.to(dtype).cuda()
    s, q = U.to_mx(x)
    rs, rq = O.to_mx(as_oracle_input(x))
    np.testing.assert_array_equal(u8(s), rs)
    np.testing.assert_array_equal(u8(q), rq)


def test_negative_underflow_and_ties(U):
    # -tiny next to a large value rounds to -0 (0x80); ties go to even
    x = torch.zeros(4, 32)
    x[0, 0] = 448.0
    x[0, 1:] = -torch.arange(1, 32) * 2.0 ** -14
    x[1] = torch.tensor([1.0 + k / 16.0 for k in range(32)])
    x[2] = torch.tensor([(2 * k + 1) * 2.0 ** -10 for k in range(32)])
    x[2, 31] = 256.0
    x[3] = -x[2]
    x = x.cuda()
    s, q = U.to_mx(x)
    rs, rq = O.to_mx(as_oracle_input(x))
    np.testing.assert_array_equal(u8(s), rs)
    np.testing.assert_array_equal(u8(q), rq)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("shape", [(32, 64), (96, 40), (512, 1000), (2048, 256)])
def test_dim1_matches_transposed_to_mx(U, dtype, shape):
    g = torch.Generator().manual_seed(7)
    x = (torch.randn(shape, generator=g) * 3).to(dtype).cuda()
    s, q = U.to_mx_dim1(x)
    assert q.shape == (shape[1], shape[0]) and s.shape == (shape[1], shape[0] // 32)
    rs, rq = O.to_mx(as_oracle_input(x).T.copy())
    np.testing.assert_array_equal(u8(s), rs)
    np.testing.assert_array_equal(u8(q), rq)


def test_blocked_scale_layout(U):
    x = (torch.randn(300, 416) * 5).to(torch.bfloat16).cuda()
    sb, qb = U.to_mx_blocked_scales(x)
    s, q = U.to_mx(x)
    assert torch.equal(qb.view(torch.uint8), q.view(torch.uint8))
    R, C = s.shape
    Rp, Cp = (R + 127) // 128 * 128, (C + 3) // 4 * 4
    pad = torch.zeros(Rp, Cp, dtype=torch.uint8, device="cuda")
    pad[:R, :C] = s
    # 128x4 atoms, row-major over (row block, col block); inside an atom
    # offset = (r % 32) * 16 + (r // 32) * 4 + c
    ref = pad.view(Rp // 128, 4, 32, Cp // 4, 4).permute(0, 3, 2, 1, 4).reshape(-1)
    assert torch.equal(sb, ref)


def test_large_rows_bandwidth_sanity(U):
    # full-size operand (16640 x 8192 bf16): compare a sampled set of rows
    x = torch.randn(16640, 8192, dtype=torch.bfloat16, device="cuda")
    s, q = U.to_mx(x)
    idx = torch.randint(0, 16640, (64,), device="cuda")
    rs, rq = O.to_mx(as_oracle_input(x[idx]))
    np.testing.assert_array_equal(u8(s[idx]), rs)
    np.testing.assert_array_equal(u8(q[idx]), rq)
