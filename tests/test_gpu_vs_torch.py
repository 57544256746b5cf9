"""Forward GEMM against torch's own MXFP8 grouped GEMM (torch._scaled_grouped_mm
on sm_100), an implementation independent of this library and of the
oracle, on the same quantised inputs.  Both accumulate the same e4m3 x e4m3
block-scaled products in fp32 and round once to bf16, so the outputs agree
to rel-L2 <= 1e-5 (most points are bit-identical; the summation order of
split tiles may move a few last bits).  Group sizes are multiples of 32 and
non-empty: the layout torch documents for the 2d x 3d case."""
import pytest
import torch

from helpers import gpu_status_clear

pytestmark = pytest.mark.gpu


def _blocked(s2d):
    """(R, C) scales -> 128x4 blocked atoms (rows padded to 128, columns to 4)."""
    R, C = s2d.shape
    Rp, Cp = -(-R // 128) * 128, -(-C // 4) * 4
    pad = torch.zeros((Rp, Cp), dtype=torch.uint8, device=s2d.device)
    pad[:R, :C] = s2d.view(torch.uint8)
    return pad.view(Rp // 128, 128, Cp // 4, 4).permute(0, 2, 1, 3).reshape(-1, 4, 32, 4).transpose(1, 2).reshape(Rp, Cp)


@pytest.mark.parametrize("E,M,N,K,offs", [
    (4, 1024, 256, 512, [128, 320, 704, 1024]),
    (2, 2048, 1024, 2048, [992, 2048]),
    (8, 4096, 512, 1024, [256, 768, 800, 1536, 2048, 2560, 3584, 4096]),
])
def test_forward_matches_torch_scaled_grouped_mm(E, M, N, K, offs):
    import kernels
    import utils
    gpu_status_clear()
    g = torch.Generator().manual_seed(E + N)
    a_s, a_q = utils.to_mx(torch.randn(M, K, generator=g).to(torch.bfloat16).cuda())
    b_s, b_q = utils.to_mx((torch.randn(E, N, K, generator=g) * 0.05).to(torch.bfloat16).cuda())
    o = torch.tensor(offs, dtype=torch.int32, device="cuda")
    ends = [0] + offs
    sa = torch.cat([_blocked(a_s[ends[i]:ends[i + 1]]) for i in range(E)]).view(torch.float8_e8m0fnu)
    sb = torch.stack([_blocked(b_s[e]).reshape(-1) for e in range(E)]).view(torch.float8_e8m0fnu)
    ref = torch._scaled_grouped_mm(a_q, b_q.transpose(-2, -1), sa, sb, offs=o, out_dtype=torch.bfloat16)
    out = kernels.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, o)
    torch.cuda.synchronize()
    rows = offs[-1]
    d = (out[:rows].float() - ref[:rows].float()).norm() / ref[:rows].float().norm()
    assert d.item() <= 1e-5, d.item()
    assert gpu_status_clear() == 0
