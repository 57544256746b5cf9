"""Expert parallelism for the MXFP8 grouped GEMMs over ``torch.distributed``.

One process per GPU.  Each rank holds its own tokens, sorted by expert (the
layout the reference's ``group_end_offsets`` describe), and the weights of the
experts it hosts.  A forward (or dgrad) grouped GEMM becomes

    counts exchange -> token all-to-all (fp8 rows + e8m0 scales)
    -> local grouped GEMM over the received segments -> all-to-all back

with NCCL moving the bytes over NVLink.  The receive buffer is source-major
(all rows from rank 0, then rank 1, ...), and within a source block it is
expert-major; ``mxgg::grouped_mm_segments`` multiplies each (source, expert)
segment by its expert's weights in place, so nothing is permuted.  The
return all-to-all mirrors the dispatch, so every rank gets its rows back in
its own order.

Placement.  With E >= world, rank r hosts experts [r*L, (r+1)*L), L = E/world.
With E < world, every expert is hosted by R = world/E ranks (replicas) and a
source rank s sends expert e's rows to replica s % R, so each replica sees the
same token count as a single GPU would.  (Splitting N across ranks instead
would all-gather every token to every rank: world times the dispatch volume
for weak-scaled token shards.)  Replicated experts sum their weight gradients
with an all-reduce over the replica group.

Nothing here synchronises the device except ``plan_dispatch``, which needs the
received counts on the host to size the NCCL transfers.
"""

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch
from torch import Tensor


class ExpertPlacement:
    """Which rank computes which expert's rows."""

    def __init__(self, world: int, n_experts: int):
        if world < 1 or n_experts < 1:
            raise ValueError(f"bad placement: world={world}, experts={n_experts}")
        self.world = world
        self.n_experts = n_experts
        if n_experts >= world:
            if n_experts % world:
                raise ValueError(f"{n_experts} experts do not divide over {world} ranks")
            self.local = n_experts // world
            self.replicas = 1
        else:
            if world % n_experts:
                raise ValueError(f"{world} ranks do not divide into replicas of {n_experts} experts")
            self.local = 1
            self.replicas = world // n_experts

    def experts_of(self, rank: int) -> List[int]:
        """Experts hosted by `rank`, in local-index order."""
        if self.replicas == 1:
            return list(range(rank * self.local, (rank + 1) * self.local))
        return [rank // self.replicas]

    def dest(self, src: int, expert: int) -> int:
        """Rank that computes the rows of `expert` held by rank `src`."""
        if self.replicas == 1:
            return expert // self.local
        return expert * self.replicas + src % self.replicas

    def local_index(self, expert: int) -> int:
        return expert % self.local if self.replicas == 1 else 0

    def replica_group(self, rank: int) -> List[int]:
        """Ranks hosting the same experts as `rank` (itself included)."""
        if self.replicas == 1:
            return [rank]
        e = rank // self.replicas
        return list(range(e * self.replicas, (e + 1) * self.replicas))


@dataclass
class DispatchPlan:
    """Sizes of one dispatch / combine pair, as seen by one rank."""

    placement: ExpertPlacement
    rank: int
    send_splits: List[int]       # rows to each rank (local rows are sorted by destination)
    recv_splits: List[int]       # rows from each rank
    seg_counts: List[int]        # rows per (source, local expert), source-major
    seg_offs: Tensor             # (world * L,) int32 cumulative ends, on the compute device
    seg_expert: Tensor           # (world * L,) int32 local expert of each segment
    rows_local: int
    rows_recv: int

    def expert_rows(self) -> List[int]:
        """Received rows per local expert (over all sources)."""
        L = self.placement.local
        return [sum(self.seg_counts[s * L + e] for s in range(self.placement.world)) for e in range(L)]


def _dist():
    import torch.distributed as dist
    return dist


def plan_dispatch(placement: ExpertPlacement, expert_counts: Sequence[int], device: torch.device,
                  group=None) -> DispatchPlan:
    """Exchange per-expert row counts and derive the all-to-all splits.

    `expert_counts[e]` is the number of this rank's rows routed to expert e;
    the rows are stored sorted by expert.  `device` is where the counts travel
    (cuda for NCCL, cpu for gloo) and where the segment tables are built.
    """
    dist = _dist()
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if world != placement.world:
        raise ValueError(f"placement for {placement.world} ranks used on {world}")
    E, L = placement.n_experts, placement.local
    if len(expert_counts) != E:
        raise ValueError(f"{len(expert_counts)} counts for {E} experts")
    send = torch.zeros(world, L, dtype=torch.int64)
    prev_dest = 0
    for e, c in enumerate(expert_counts):
        if c < 0:
            raise ValueError(f"negative count for expert {e}")
        d = placement.dest(rank, e)
        if d < prev_dest:
            raise AssertionError("destinations must be monotone in the expert index")
        prev_dest = d
        send[d, placement.local_index(e)] += int(c)
    recv = torch.empty_like(send, device=device)
    dist.all_to_all_single(recv, send.to(device), group=group)
    recv = recv.cpu()
    seg_counts = recv.reshape(-1).tolist()
    offs = torch.tensor(seg_counts, dtype=torch.int64).cumsum(0).to(torch.int32)
    expert = torch.arange(L, dtype=torch.int32).repeat(world)
    return DispatchPlan(placement=placement, rank=rank, send_splits=send.sum(1).tolist(),
                        recv_splits=recv.sum(1).tolist(), seg_counts=seg_counts, seg_offs=offs.to(device),
                        seg_expert=expert.to(device), rows_local=int(send.sum()), rows_recv=int(recv.sum()))


def _a2a_rows(x: Tensor, out_rows: int, out_splits: List[int], in_splits: List[int], group=None) -> Tensor:
    """All-to-all of the rows of a 2-D tensor (any dtype, moved as bytes)."""
    dist = _dist()
    row_bytes = x.element_size() * math.prod(x.shape[1:])
    xb = x.contiguous().view(torch.uint8).reshape(x.shape[0], row_bytes)
    out = torch.empty((out_rows, row_bytes), dtype=torch.uint8, device=x.device)
    dist.all_to_all_single(out, xb, out_splits, in_splits, group=group)
    return out.view(x.dtype).reshape(out_rows, *x.shape[1:])


def dispatch(plan: DispatchPlan, *tensors: Tensor, group=None) -> List[Tensor]:
    """Send each tensor's rows (this rank's, sorted by expert) to their experts' ranks."""
    return [_a2a_rows(t, plan.rows_recv, plan.recv_splits, plan.send_splits, group) for t in tensors]


def combine(plan: DispatchPlan, y: Tensor, group=None) -> Tensor:
    """Return computed rows to the ranks that own them, in their original order."""
    return _a2a_rows(y, plan.rows_local, plan.send_splits, plan.recv_splits, group)


def ep_grouped_mm(plan: DispatchPlan, a_q: Tensor, a_s: Tensor, w_q: Tensor, w_s: Tensor,
                  out_dtype: torch.dtype = torch.bfloat16, group=None) -> Tensor:
    """Expert-parallel forward / dgrad: dispatch, local segment GEMM, combine.

    a_q (rows_local, K) e4m3 and a_s (rows_local, K/32) are this rank's rows
    sorted by expert; w_q (L, N, K) / w_s (L, N, K/32) are the hosted experts.
    Returns (rows_local, N) in this rank's row order.
    """
    from .ops import grouped_mm_segments_op
    recv_q, recv_s = dispatch(plan, a_q, a_s, group=group)
    y = grouped_mm_segments_op(recv_q, w_q, recv_s, w_s, plan.seg_offs, plan.seg_expert, out_dtype)
    return combine(plan, y, group=group)


def replica_allreduce(placement: ExpertPlacement, t: Tensor, groups: Optional[dict] = None) -> Tensor:
    """Sum a hosted expert's weight gradient over its replicas (no-op without replicas).

    `groups` maps a replica-rank tuple to its process group; build it once with
    `replica_groups(placement)` on every rank (group creation is collective).
    """
    if placement.replicas == 1:
        return t
    dist = _dist()
    g = groups[tuple(placement.replica_group(dist.get_rank()))]
    dist.all_reduce(t, group=g)
    return t


def replica_groups(placement: ExpertPlacement) -> dict:
    """Process groups of the replica sets (collective: call on every rank)."""
    dist = _dist()
    out = {}
    if placement.replicas == 1:
        return out
    for e in range(placement.n_experts):
        ranks = tuple(range(e * placement.replicas, (e + 1) * placement.replicas))
        out[ranks] = dist.new_group(list(ranks))
    return out
