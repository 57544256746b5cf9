"""Expert-parallel grouped GEMM on 2 GPUs (skipped with fewer): NCCL
all-to-all dispatch/combine, and the fused path (peer-memory dispatch,
combine inside the GEMM epilogue).

Each rank quantises its own tokens (sorted by expert, seeded per rank) and
holds the full weights only to build the check: the expert-parallel result
(dispatch -> segment GEMM on the hosting rank -> combine) must equal the
single-GPU grouped GEMM of the same rows.  With whole-tile scheduling every
output element is the same fp32 MMA chain in both, so the check is bit-exact.
"""
import os

import pytest
import torch

from helpers import run_ranks

pytestmark = pytest.mark.gpu


def _worker(rank, world, store, q, E, impl, align, big=False):
    import datetime
    import torch.distributed as dist
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method="file://" + store, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
        import kernels
        import mxgg
        import utils
        from mxgg.ep import ExpertPlacement, ep_grouped_mm, plan_dispatch
        mxgg.set_schedule(mxgg._lib.SCHED_TILES, 0)
        dev = torch.device("cuda", rank)
        N, K = (1024, 1024) if big else (384, 512)
        pl = ExpertPlacement(world, E)
        gw = torch.Generator().manual_seed(7)
        W = torch.randn(E, N, K, generator=gw).to(torch.bfloat16).to(dev)
        fp4 = impl.endswith("fp4")
        w_s, w_q = utils.to_mx(W, elem_dtype=torch.float4_e2m1fn_x2 if fp4 else torch.float8_e4m3fn)
        g = torch.Generator().manual_seed(11 + rank)
        counts = [int(c) * align * (16 if big else 1) for c in torch.randint(0, 9, (E,), generator=g)]
        if rank == 1:
            counts[-1] = 0
        rows = sum(counts)
        A = torch.randn(rows, K, generator=g).to(torch.bfloat16).to(dev)
        a_s, a_q = utils.to_mx(A)
        offs = torch.tensor(counts, dtype=torch.int64).cumsum(0).to(torch.int32).to(dev)
        ref = kernels.triton_mxfp8_grouped_mm(a_q, w_q, a_s, w_s, offs, out_dtype=torch.float32)
        mine = pl.experts_of(rank)
        wq_mine = w_q.view(torch.uint8)[mine].contiguous().view(w_q.dtype)   # (no index kernels for 4-bit dtypes)
        ws_mine = w_s[mine].contiguous()
        if impl.startswith("nccl"):
            plan = plan_dispatch(pl, counts, dev)
            got = ep_grouped_mm(plan, a_q, a_s, wq_mine, ws_mine,
                                out_dtype=torch.float32)
        else:
            from mxgg.ep import FusedExpertParallel
            cap = 8 * 32 * E * (16 if big else 1)             # most rows any rank can hold
            fused = FusedExpertParallel(pl, max_recv_rows=world * cap, max_local_rows=cap, max_k=K, max_n=N)
            plan = fused.plan(counts)
            # a first call on other rows, then the checked one: stale rows left
            # in the shared buffers by the first call cannot pass for fresh ones
            A0 = torch.randn(rows, K, generator=g).to(torch.bfloat16).to(dev)
            a0_s, a0_q = utils.to_mx(A0)
            first = fused.grouped_mm(plan, a0_q, a0_s, wq_mine, ws_mine, out_dtype=torch.float32).clone()
            ref0 = kernels.triton_mxfp8_grouped_mm(a0_q, w_q, a0_s, w_s, offs, out_dtype=torch.float32)
            got = fused.grouped_mm(plan, a_q, a_s, wq_mine, ws_mine, out_dtype=torch.float32).clone()
            torch.cuda.synchronize()
            if not torch.equal(first, ref0):
                got = first          # report the first call's mismatch below
        torch.cuda.synchronize()
        ok = got.shape == ref.shape and torch.equal(got, ref)
        st = mxgg.device_status(clear=True)
        if not impl.startswith("nccl"):
            fused.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok" if ok and st == 0 else f"mismatch (status {st}): "
               f"max err {(got.float() - ref.float()).abs().max().item() if got.shape == ref.shape else got.shape}"))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("impl,align", [("nccl", 32), ("fused", 32), ("fused", 16), ("fused-fp4", 32)])
@pytest.mark.parametrize("E", [4, 1])
def test_ep_grouped_mm_two_ranks(E, impl, align):
    """align 32: peers' output blocks travel through inboxes; align 16: some
    segments start off the 32-row grid and rows are stored in place."""
    results = run_ranks(_worker, 2, E, impl, align)
    for r in range(2):
        assert results.get(r) == "ok", results.get(r)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_fused_full_grid():
    """A GEMM that fills every SM while it streams in peers' rows: the
    senders' flags must still get through (they are stream memory operations,
    not kernels that would need a free SM)."""
    results = run_ranks(_worker, 2, 4, "fused", 32, True)
    for r in range(2):
        assert results.get(r) == "ok", results.get(r)
