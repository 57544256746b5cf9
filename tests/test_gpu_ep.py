"""Expert-parallel grouped GEMM on 2 GPUs over NCCL (skipped with fewer).

Each rank quantises its own tokens (sorted by expert, seeded per rank) and
holds the full weights only to build the check: the expert-parallel result
(dispatch -> segment GEMM on the hosting rank -> combine) must equal the
single-GPU grouped GEMM of the same rows.  With whole-tile scheduling every
output element is the same fp32 MMA chain in both, so the check is bit-exact.
"""
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, E, port, q):
    import datetime
    import torch.distributed as dist
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        torch.cuda.set_device(rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        import kernels
        import mxgg
        import utils
        from mxgg.ep import ExpertPlacement, ep_grouped_mm, plan_dispatch
        mxgg.set_schedule(mxgg._lib.SCHED_TILES, 0)
        dev = torch.device("cuda", rank)
        N, K = 384, 512
        pl = ExpertPlacement(world, E)
        gw = torch.Generator().manual_seed(7)
        W = torch.randn(E, N, K, generator=gw).to(torch.bfloat16).to(dev)
        w_s, w_q = utils.to_mx(W)
        g = torch.Generator().manual_seed(11 + rank)
        counts = [int(c) * 32 for c in torch.randint(0, 9, (E,), generator=g)]
        if rank == 1:
            counts[-1] = 0
        rows = sum(counts)
        A = torch.randn(rows, K, generator=g).to(torch.bfloat16).to(dev)
        a_s, a_q = utils.to_mx(A)
        offs = torch.tensor(counts, dtype=torch.int64).cumsum(0).to(torch.int32).to(dev)
        ref = kernels.triton_mxfp8_grouped_mm(a_q, w_q, a_s, w_s, offs, out_dtype=torch.float32)
        plan = plan_dispatch(pl, counts, dev)
        mine = pl.experts_of(rank)
        got = ep_grouped_mm(plan, a_q, a_s, w_q[mine].contiguous(), w_s[mine].contiguous(),
                            out_dtype=torch.float32)
        torch.cuda.synchronize()
        ok = got.shape == ref.shape and torch.equal(got, ref)
        st = mxgg.device_status(clear=True)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok" if ok and st == 0 else f"mismatch (status {st}): "
               f"max err {(got.float() - ref.float()).abs().max().item() if got.shape == ref.shape else got.shape}"))
    except Exception:
        import traceback
        q.put((rank, traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("E", [4, 1])
def test_ep_grouped_mm_two_ranks(E):
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, E, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(world):
            r, msg = q.get(timeout=300)
            results[r] = msg
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(world):
        assert results.get(r) == "ok", results.get(r)
