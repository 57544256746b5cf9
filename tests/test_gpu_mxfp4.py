"""MXFP4 (e2m1) weights on the GPU against the oracle.

Quantiser: bytes bit-exact with the oracle's e2m1 restatement (FLOOR scaling
with emax 2, RNE on the e2m1 grid, saturation to +-6, NaN -> +6, element 2i
in the low nibble).  GEMM: e4m3 activations x e2m1 weights on the
kind::mxf8f6f4 tensor-core path, rel-L2 <= 1e-3 (bf16 out, both sides rounded
to bf16) / <= 1e-5 (fp32 out) against dequantise-then-fp32-matmul.
"""
import numpy as np
import pytest
import torch

from helpers import O, bf16_round, f32, gpu_status_clear, u8

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status():
    gpu_status_clear()
    yield
    assert gpu_status_clear() == 0, "a device-side wait timed out"


def _edge_rows(C):
    rows = []
    z = np.zeros(C, np.float32)
    rows.append(z)                                           # all zeros -> scale 0
    r = np.zeros(C, np.float32)
    r[:32] = [.25, .75, 1.25, 1.75, 2.5, 3.5, 5.0, -5.0] * 4   # ties at scale 1 (amax 5 -> e=2)
    rows.append(r)
    r = np.full(C, 1e-30, np.float32)                        # tiny values, subnormal products
    r[3] = 3e-30
    rows.append(r)
    r = np.linspace(-1e30, 1e30, C).astype(np.float32)       # huge values
    rows.append(r)
    r = np.ones(C, np.float32)
    r[5] = np.inf
    r[40] = -np.inf
    r[70] = np.nan
    rows.append(r)                                           # inf / NaN blocks
    return np.stack(rows)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
def test_quantize_e2m1_bit_exact(dtype):
    import utils
    g = torch.Generator().manual_seed(5)
    C = 256
    x = torch.randn(64, C, generator=g) * torch.logspace(-3, 3, 64)[:, None]
    x = torch.cat([x, torch.from_numpy(_edge_rows(C))]).to(dtype)
    s, q = utils.to_mx(x.cuda(), elem_dtype=torch.float4_e2m1fn_x2)
    torch.cuda.synchronize()
    assert q.dtype == torch.float4_e2m1fn_x2 and q.shape == (x.shape[0], C // 2)
    rs, rq = O.to_mx(x.float().numpy(), elem="e2m1")
    assert np.array_equal(u8(s), rs)
    assert np.array_equal(u8(q), O.pack_e2m1(rq))


def _make(E, M, N, K, offs, seed):
    import utils
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    W = (torch.randn(E, N, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
    a_s, a_q = utils.to_mx(A)
    w_s, w_q = utils.to_mx(W, elem_dtype=torch.float4_e2m1fn_x2)
    return a_s, a_q, w_s, w_q, torch.tensor(offs, dtype=torch.int32, device="cuda")


def _oracle(a_q, a_s, w_q, w_s, offs):
    wn = O.unpack_e2m1(u8(w_q))
    return O.grouped_mm(u8(a_q), u8(a_s), wn, u8(w_s), offs.cpu().numpy(), acc=np.float32, b_elem="e2m1")


def _check(out, ref, out_dtype):
    valid = ~np.isnan(ref)
    if out_dtype == torch.float32:
        assert O.rel_l2(f32(out)[valid], ref[valid]) <= 1e-5
    else:
        assert O.rel_l2(f32(out)[valid], bf16_round(ref)[valid]) <= 1e-3


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("tile_m,tile_n", [(256, 256), (128, 128), (256, 128)])
@pytest.mark.parametrize("E,M,N,K,offs", [
    (4, 1024, 256, 512, [128, 128, 640, 1024]),        # an empty group, ragged edges
    (2, 2048, 640, 1024, [736, 2048]),                 # N tail
    (1, 512, 256, 4096, [512]),                        # long contraction
])
def test_grouped_mm_e2m1_weights(out_dtype, tile_m, tile_n, E, M, N, K, offs):
    import kernels
    import mxgg
    a_s, a_q, w_s, w_q, o = _make(E, M, N, K, offs, seed=E + K)
    mxgg.set_tile_config(tile_m, tile_n, 0)
    try:
        out = kernels.triton_mxfp8_grouped_mm(a_q, w_q, a_s, w_s, o, out_dtype=out_dtype)
        torch.cuda.synchronize()
    finally:
        mxgg.set_tile_config(0, 0, 0)
    _check(out, _oracle(a_q, a_s, w_q, w_s, o), out_dtype)


def test_e2m1_rejects_k_tail():
    import kernels
    from mxgg import _lib
    a_s, a_q, w_s, w_q, o = _make(1, 256, 256, 96, [256], seed=1)
    with pytest.raises(_lib.MxggError, match="K % 128"):
        kernels.triton_mxfp8_grouped_mm(a_q, w_q, a_s, w_s, o)
