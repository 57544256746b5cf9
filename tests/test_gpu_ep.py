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
            # "fused-pieces": peers' rows travel in pieces of >= 64 rows, each flagged on its own
            plan = fused.plan(counts, piece_rows=64 if impl == "fused-pieces" else 2048)
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
@pytest.mark.parametrize("impl,align", [("nccl", 32), ("fused", 32), ("fused", 16), ("fused-fp4", 32),
                                        ("fused-pieces", 32), ("fused-pieces", 16)])
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


def _replica_worker(rank, world, store, q, dtype_name):
    import datetime
    import torch.distributed as dist
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method="file://" + store, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
        import mxgg
        from mxgg.ep import ExpertPlacement, ReplicaSum
        dev = torch.device("cuda", rank)
        dt = getattr(torch, dtype_name)
        shape = (1, 384, 2080)                     # not a multiple of the ranks' shares
        rs = ReplicaSum(2 * 384 * 2080 * 4)
        msgs = []
        for E in [e for e in (1, 2, 4) if world % e == 0 and world // e > 1]:
            pl = ExpertPlacement(world, E)
            for inplace in (True, False):
                g = torch.Generator(device=dev).manual_seed(100 * E + rank)
                x = torch.randn(shape, generator=g, device=dev).to(dt)
                t = rs.buffer(shape, dt) if inplace else torch.empty(shape, dtype=dt, device=dev)
                t.copy_(x)
                rs.sum_(pl, t)
                allx = [torch.empty_like(x) for _ in range(world)]
                dist.all_gather(allx, x)
                want = torch.zeros(shape, dtype=torch.float32, device=dev)
                for r in pl.replica_group(rank):           # fp32, replica order, one rounding
                    want += allx[r].float()
                want = want.to(dt)
                # every replica holds the same bits: compare with the group's first replica
                got_all = [torch.empty_like(x) for _ in range(world)]
                dist.all_gather(got_all, t.contiguous())
                first = got_all[pl.replica_group(rank)[0]]
                if not torch.equal(t, want) or not torch.equal(t, first):
                    msgs.append(f"E={E} inplace={inplace}: max err {(t.float() - want.float()).abs().max().item()}")
        st = mxgg.device_status(clear=True)
        torch.cuda.synchronize()
        rs.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok" if not msgs and st == 0 else f"status {st}; " + "; ".join(msgs)))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("dtype_name", ["bfloat16", "float32"])
def test_replica_sum_matches_fp32_sum(dtype_name):
    """The peer-memory replica sum equals the fp32 sum of every replica in
    replica order, rounded once, and leaves all replicas bit-identical
    (2 GPUs: one group of 2; 4 GPUs: groups of 4 and of 2; 8 GPUs: 8, 4, 2)."""
    n = torch.cuda.device_count()
    world = 8 if n >= 8 else 4 if n >= 4 else 2
    results = run_ranks(_replica_worker, world, dtype_name)
    for r in range(world):
        assert results.get(r) == "ok", results.get(r)


def _replica_wgrad_worker(rank, world, store, q, N, K):
    import datetime
    import torch.distributed as dist
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", init_method="file://" + store, rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", rank))
        import mxgg
        import utils
        from mxgg.ep import ExpertPlacement, ReplicaSum
        dev = torch.device("cuda", rank)
        M = 1024
        pl = ExpertPlacement(world, 1)                       # one expert, `world` replicas
        g = torch.Generator(device=dev).manual_seed(40 + rank)
        go = torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16)
        x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
        go_s, go_q = utils.to_mx_dim1(go)
        x_s, x_q = utils.to_mx_dim1(x)
        offs = torch.tensor([M], dtype=torch.int32, device=dev)
        mine = mxgg.ops.wgrad(go_q, go_s, x_q, x_s, offs, torch.bfloat16)   # one launch, default schedule
        rs = ReplicaSum(N * K * 2)
        split = rs.split_rows(1, N, K)
        msgs = []
        for it in range(2):                                  # the second call reuses the buffer
            got = rs.wgrad_sum(pl, go_q, go_s, x_q, x_s, offs)
            allg = [torch.empty_like(mine) for _ in range(world)]
            dist.all_gather(allg, mine)
            want = torch.zeros_like(mine, dtype=torch.float32)
            for r in pl.replica_group(rank):
                want += allg[r].float()
            if not torch.equal(got, want.to(torch.bfloat16)):
                msgs.append(f"call {it}: max err {(got.float() - want).abs().max().item()}")
        st = mxgg.device_status(clear=True)
        torch.cuda.synchronize()
        rs.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok" if not msgs and st == 0 else f"split {split}, status {st}; " + "; ".join(msgs)))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("N,K", [(5120, 5120), (1024, 768)])
def test_replica_wgrad_sum_overlapped(N, K):
    """ReplicaSum.wgrad_sum: the gradient computed in two launches (N=K=5120:
    the first part's replica sum overlaps the second part's GEMM) or one
    (a small grid), summed over the replicas, equals the fp32 sum of every
    replica's one-launch gradient in replica order, rounded once."""
    results = run_ranks(_replica_wgrad_worker, 2, N, K)
    for r in range(2):
        assert results.get(r) == "ok", results.get(r)
