"""MoE layer forward on the GPU.

1 GPU: against an fp32 torch reference of the same layer (unquantised bf16
inputs and weights): SQNR >= 20 dB with MXFP8 weights, >= 10 dB with MXFP4
weights (two quantised GEMMs in a row).  The gathered quantiser is checked
bit-exact against to_mx of the gathered rows.
2 GPUs: the expert-parallel layer equals the single-GPU layer bit for bit
(whole-tile schedule) for MXFP8 and MXFP4 weights.
"""
import os

import pytest
import torch

from helpers import O, f32, gpu_status_clear, run_ranks

pytestmark = pytest.mark.gpu


def _weights(E, d_model, d_ff, seed=3):
    g = torch.Generator().manual_seed(seed)
    up = (torch.randn(E, d_ff, d_model, generator=g) * d_model ** -0.5).to(torch.bfloat16)
    down = (torch.randn(E, d_model, d_ff, generator=g) * d_ff ** -0.5).to(torch.bfloat16)
    return up, down


def _reference(x, logits, up, down):
    from mxgg.moe import route_top2
    e, w = route_top2(logits)
    xf = x.float()
    out = torch.zeros_like(xf)
    for k in range(2):
        for ex in range(up.shape[0]):
            m = e[:, k] == ex
            if m.any():
                h = xf[m] @ up[ex].float().t()
                out[m] += w[m, k, None] * (h @ down[ex].float().t())
    return out


@pytest.fixture(autouse=True)
def _status():
    gpu_status_clear()
    yield
    assert gpu_status_clear() == 0, "a device-side wait timed out"


def test_quantize_gather_bit_exact():
    import numpy as np
    import utils
    from mxgg.moe import quantize_gather
    g = torch.Generator().manual_seed(2)
    x = torch.randn(100, 256, generator=g).to(torch.bfloat16).cuda()
    idx = torch.tensor([5, -1, 99, 0, 0, -1, 42, 7] * 8, dtype=torch.int32).cuda()
    s, q = quantize_gather(x, idx)
    rows = torch.where(idx[:, None] >= 0, x[idx.clamp(min=0).long()], torch.zeros_like(x[:1]))
    rs, rq = utils.to_mx(rows)
    torch.cuda.synchronize()
    assert torch.equal(s, rs) and torch.equal(q.view(torch.uint8), rq.view(torch.uint8))


def test_combine_top2_matches_torch():
    from mxgg.moe import combine_top2, dispatch_layout, route_top2
    g = torch.Generator().manual_seed(4)
    T, E, N = 300, 6, 512
    e, w = route_top2(torch.randn(T, E, generator=g).cuda())
    lay = dispatch_layout(e, E)
    y = torch.randn(sum(lay.counts), N, generator=g).to(torch.bfloat16).cuda()
    got = combine_top2(y, lay, w)
    ref = (y[lay.pair_pos.reshape(-1)].float().reshape(T, 2, N) * w[..., None]).sum(1)
    torch.cuda.synchronize()
    # fp32 sums that may differ by one fused multiply-add rounding, then bf16
    torch.testing.assert_close(got.float(), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("fp4,min_sqnr", [(False, 20.0), (True, 10.0)])
def test_moe_layer_single_gpu(fp4, min_sqnr):
    from mxgg.moe import MoELayer
    E, T, d_model, d_ff = 4, 512, 256, 512
    up, down = _weights(E, d_model, d_ff)
    g = torch.Generator().manual_seed(9)
    x = torch.randn(T, d_model, generator=g).to(torch.bfloat16).cuda()
    logits = torch.randn(T, E, generator=g).cuda()
    layer = MoELayer(up.cuda(), down.cuda(), E, weights_fp4=fp4)
    out = layer.forward(x, logits)
    torch.cuda.synchronize()
    ref = _reference(x, logits, up.cuda(), down.cuda())
    sqnr = O.compute_error(f32(ref), f32(out))
    assert sqnr >= min_sqnr, sqnr


def _worker(rank, world, store, q, fp4):
    import datetime
    import torch.distributed as dist
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method="file://" + store, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
        import mxgg
        from mxgg.ep import ExpertPlacement, FusedExpertParallel
        from mxgg.moe import MoELayer
        mxgg.set_schedule(mxgg._lib.SCHED_TILES, 0)
        E, T, d_model, d_ff = 4, 384, 256, 512
        up, down = _weights(E, d_model, d_ff)
        g = torch.Generator().manual_seed(20 + rank)
        x = torch.randn(T, d_model, generator=g).to(torch.bfloat16).cuda()
        logits = torch.randn(T, E, generator=g).cuda()
        single = MoELayer(up.cuda(), down.cuda(), E, weights_fp4=fp4).forward(x, logits)
        pl = ExpertPlacement(world, E)
        mine = pl.experts_of(rank)
        cap = 2 * T + 32 * E
        ep = FusedExpertParallel(pl, max_recv_rows=world * cap, max_local_rows=cap, max_k=d_ff, max_n=d_ff)
        layer = MoELayer(up[mine].cuda(), down[mine].cuda(), E, weights_fp4=fp4, placement=pl, ep=ep)
        # a first call on other tokens, then the checked one: stale rows in the
        # shared buffers cannot pass for fresh ones
        x0 = torch.randn(T, d_model, generator=g).to(torch.bfloat16).cuda()
        first = layer.forward(x0, logits).clone()
        single0 = MoELayer(up.cuda(), down.cuda(), E, weights_fp4=fp4).forward(x0, logits)
        got = layer.forward(x, logits).clone()
        torch.cuda.synchronize()
        ok = torch.equal(got, single) and torch.equal(first, single0)
        st = mxgg.device_status(clear=True)
        ep.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok" if ok and st == 0 else
               f"mismatch (status {st}): max err {(got.float() - single.float()).abs().max().item()}"))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("fp4", [False, True])
def test_moe_layer_expert_parallel_two_ranks(fp4):
    results = run_ranks(_worker, 2, fp4)
    for r in range(2):
        assert results.get(r) == "ok", results.get(r)
