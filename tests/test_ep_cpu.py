"""Expert-parallel host logic on CPU: placement, the counts exchange, dispatch
and combine, run as gloo process groups (world 2 and 4).

A stand-in for the local GEMM multiplies every received row by (1 + its
expert's global index), read from the segment tables, so the round trip
checks that rows reach the right expert and come back in their owner's order.
"""
import pytest
import torch
import torch.distributed as dist
from helpers import run_ranks
from mxgg.ep import ExpertPlacement, combine, dispatch, plan_dispatch, replica_allreduce, replica_groups


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("E", [1, 2, 4, 8, 16, 64])
def test_placement(world, E):
    if E >= world and E % world or E < world and world % E:
        with pytest.raises(ValueError):
            ExpertPlacement(world, E)
        return
    pl = ExpertPlacement(world, E)
    hosts = {e: [r for r in range(world) if e in pl.experts_of(r)] for e in range(E)}
    assert all(len(h) == pl.replicas for h in hosts.values())
    for s in range(world):
        dests = [pl.dest(s, e) for e in range(E)]
        assert dests == sorted(dests)                       # rows sorted by expert are sorted by rank
        for e, d in enumerate(dests):
            assert e in pl.experts_of(d)
            assert pl.experts_of(d)[pl.local_index(e)] == e
            assert d in pl.replica_group(d)
    if pl.replicas > 1:
        # every replica of an expert receives from the same number of sources
        for e in range(E):
            got = [sum(pl.dest(s, e) == r for s in range(world)) for r in hosts[e]]
            assert got == [world // pl.replicas] * pl.replicas


def _worker(rank, world, store, q, E):
    try:
        dist.init_process_group("gloo", init_method="file://" + store, rank=rank, world_size=world)
        pl = ExpertPlacement(world, E)
        g = torch.Generator().manual_seed(100 + rank)
        counts = [int(c) * 32 for c in torch.randint(0, 4, (E,), generator=g)]
        if rank == 0:
            counts[0] = 0                                    # an empty (source, expert) segment
        rows = sum(counts)
        K = 64
        expert_of_row = torch.repeat_interleave(torch.arange(E), torch.tensor(counts, dtype=torch.int64))
        x = torch.randn(rows, K, generator=g).to(torch.bfloat16)
        tag = torch.stack([torch.full((rows,), rank), torch.arange(rows), expert_of_row], 1).to(torch.int32)
        plan = plan_dispatch(pl, counts, torch.device("cpu"))
        assert plan.rows_local == rows
        rx, rtag = dispatch(plan, x, tag)
        assert rx.shape == (plan.rows_recv, K)
        # segments: source-major, then local expert; every row is where the tables say
        offs = [0] + plan.seg_offs.tolist()
        mine = pl.experts_of(rank)
        y = torch.empty_like(rx)
        for s_i in range(len(plan.seg_counts)):
            lo, hi = offs[s_i], offs[s_i + 1]
            src, le = divmod(s_i, pl.local)
            assert int(plan.seg_expert[s_i]) == le
            e = mine[le]
            if hi > lo:
                assert torch.all(rtag[lo:hi, 0] == src)
                assert torch.all(rtag[lo:hi, 2] == e)
            y[lo:hi] = (rx[lo:hi].float() * (1 + e)).to(torch.bfloat16)
        back = combine(plan, y)
        assert back.shape == x.shape
        want = (x.float() * (1 + expert_of_row[:, None].float())).to(torch.bfloat16)
        assert torch.equal(back, want)
        # replicated experts: weight gradients are summed over the replica set
        groups = replica_groups(pl)
        t = torch.full((4,), float(rank))
        replica_allreduce(pl, t, groups)
        assert torch.all(t == float(sum(pl.replica_group(rank))))
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as ex:  # pragma: no cover - reported through the queue
        import traceback
        q.put((rank, traceback.format_exc()))
        raise


@pytest.mark.parametrize("world,E", [(2, 4), (2, 2), (2, 1), (4, 8), (4, 2)])
def test_dispatch_combine_gloo(world, E):
    results = run_ranks(_worker, world, E, timeout=120)
    for r in range(world):
        assert results.get(r) == "ok", results.get(r)
