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


# ----------------------------------------------------------------------------
# Fused path: peer-memory dispatch, combine fused into the GEMM epilogue.
# ----------------------------------------------------------------------------
@dataclass
class _Segments:
    offs: Tensor                 # int32 cumulative ends of the segments (rows of the A operand)
    expert: Tensor               # local expert of each segment
    dst: Tensor                  # rank that owns each segment's rows
    dst_row: Tensor              # first row of the segment in its owner's output


@dataclass
class FusedPlan:
    """Routing of one fused expert-parallel call, as seen by one rank.

    The rows a rank routes to its own experts never move: the "self" GEMM
    reads them from the caller's tensor (rows [self_row, self_row +
    self_rows)) while the other ranks' rows are in flight.  The receive
    buffer holds only peers' rows, source-major, then local expert."""

    rows_local: int
    rows_recv: int               # rows received from peers
    copies: List[tuple]          # (dest rank, first row there, first local row, rows), dest != this rank
    self_row: int
    self_rows: int
    self_seg: _Segments          # L segments over the self rows
    remote_seg: _Segments        # world * L segments over the receive buffer (own source: empty)
    dst_rows: List[int]          # local rows of every rank (the output buffers' heights)
    inbox_ok: bool               # every segment starts on a 32-row boundary: peers' blocks go by inbox
    remote_blocks: Tensor        # this rank's 32-row blocks computed by peers (unpacked from its inbox)


class FusedExpertParallel:
    """Expert-parallel forward / dgrad over NVLink peer memory.

    Collective to construct (it allocates and maps the shared buffers).  Per
    call (`grouped_mm`):

    1. each rank starts pushing its rows for rank d straight into d's receive
       buffer (one copy-engine ``cudaMemcpyAsync`` per peer, on parallel
       streams) and, meanwhile, multiplies the rows it routed to its own
       experts where they lie;
    2. a cross-GPU barrier, then ``mxgg_grouped_mm_ep`` multiplies the
       received segments and sends each output block to the rank that owns
       its rows as the tile finishes (TMA stores for its own rows; 2 KB bulk
       copies into the owner's inbox for peers'), so the return trip overlaps
       the math tile by tile;
    3. a second barrier, then each rank unpacks its inbox into its output.

    The returned tensor is a view of this rank's shared output buffer: use it
    before the next call.
    """

    def __init__(self, placement: ExpertPlacement, max_recv_rows: int, max_local_rows: int, max_k: int, max_n: int,
                 group=None):
        from .peer import PeerBuffer
        dist = _dist()
        self.placement = placement
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world != placement.world:
            raise ValueError("placement and process group disagree on the world size")
        if self.world > 8:
            raise ValueError("the fused path reaches at most 8 ranks (one NVLink domain)")
        self.max_recv_rows, self.max_local_rows = int(max_recv_rows), int(max_local_rows)
        self.max_k, self.max_n = int(max_k), int(max_n)
        self.recv_a = PeerBuffer(max(self.max_recv_rows * self.max_k, 256), group)
        self.recv_s = PeerBuffer(max(self.max_recv_rows * self.max_k // 32, 256), group)
        self.out = PeerBuffer(max(self.max_local_rows * self.max_n * 4, 256), group)
        self.inbox = PeerBuffer(max(self.max_local_rows * self.max_n * 4, 256), group)
        self.flags = PeerBuffer(256, group)
        self.epoch = 0
        self._streams = [torch.cuda.Stream() for _ in range(self.world)]
        self._pending = []
        # every rank's capacities, so a plan that overflows any of them fails on all ranks alike
        caps = [None] * self.world
        dist.all_gather_object(caps, (self.max_recv_rows, self.max_local_rows), group=group)
        self._caps = caps

    def close(self) -> None:
        for b in (self.recv_a, self.recv_s, self.out, self.inbox, self.flags):
            b.close()

    # -------------------------------------------------------------- planning
    def plan(self, expert_counts: Sequence[int], placement: Optional[ExpertPlacement] = None) -> FusedPlan:
        """Collective: all-gather every rank's per-expert counts and derive the
        copies, segment tables and output heights.  The shared buffers do not
        depend on the placement, so one instance serves several (`placement`
        overrides the constructor's for this plan)."""
        dist = _dist()
        pl, world, rank = placement or self.placement, self.world, self.rank
        if pl.world != world:
            raise ValueError("placement and process group disagree on the world size")
        E = pl.n_experts
        dev = torch.device("cuda", torch.cuda.current_device())
        mine = torch.tensor([int(c) for c in expert_counts], dtype=torch.int64, device=dev)
        if mine.numel() != E or bool((mine < 0).any()):
            raise ValueError("expert_counts must hold E non-negative counts")
        allc = torch.empty(world, E, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(allc, mine, group=self.group)
        C = allc.tolist()                                     # C[s][e], one device sync
        # rows rank s sends to rank d, and where they start in s's local order
        send = [[0] * world for _ in range(world)]
        start = [[0] * world for _ in range(world)]
        seen = [[False] * world for _ in range(world)]
        for s in range(world):
            row = 0
            for e in range(E):
                d = pl.dest(s, e)
                if not seen[s][d]:
                    start[s][d], seen[s][d] = row, True
                send[s][d] += C[s][e]
                row += C[s][e]
        # receive layout of rank d: peers only, source-major, then local expert
        recv_off = [[sum(send[s2][d] for s2 in range(s) if s2 != d) for d in range(world)] for s in range(world)]
        copies = [(d, recv_off[rank][d], start[rank][d], send[rank][d])
                  for d in range(world) if d != rank and send[rank][d]]
        mine_e = pl.experts_of(rank)
        i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)  # noqa: E731

        def segments(sources):
            offs, expert, dsts, first = [], [], [], []
            total = 0
            for s in range(world):
                for le, e in enumerate(mine_e):
                    rows = C[s][e] if (s in sources and pl.dest(s, e) == rank) else 0
                    total += rows
                    offs.append(total)
                    expert.append(le)
                    dsts.append(s)
                    first.append(sum(C[s][:e]))
            return total, _Segments(i32(offs), i32(expert), i32(dsts), i32(first))

        rows_recv, remote_seg = segments([s for s in range(world) if s != rank])
        self_rows, self_seg = segments([rank])
        for d in range(world):
            need_recv = sum(send[s][d] for s in range(world) if s != d)
            if need_recv > self._caps[d][0] or sum(C[d]) > self._caps[d][1]:
                raise ValueError(f"fused EP buffers of rank {d} too small: {need_recv} received / {sum(C[d])} "
                                 f"local rows for {self._caps[d][0]} / {self._caps[d][1]}")
        inbox_ok = all(c % 32 == 0 for row in C for c in row)
        blocks, row = [], 0
        for e in range(E):
            if pl.dest(rank, e) != rank:
                blocks.extend(range(row // 32, (row + C[rank][e]) // 32))
            row += C[rank][e]
        return FusedPlan(rows_local=sum(C[rank]), rows_recv=rows_recv, copies=copies, self_row=start[rank][rank],
                         self_rows=self_rows, self_seg=self_seg, remote_seg=remote_seg,
                         dst_rows=[sum(C[d]) for d in range(world)], inbox_ok=inbox_ok,
                         remote_blocks=i32(blocks if inbox_ok else []))

    # ---------------------------------------------------------------- calls
    def barrier(self) -> None:
        """Cross-GPU barrier on the current stream (bounded wait on the device)."""
        import ctypes
        from . import _lib
        self.epoch += 1
        arr = (ctypes.c_void_p * self.world)(*self.flags.ptrs)
        _lib.check(_lib.load().mxgg_peer_barrier(arr, self.world, self.rank, self.epoch,
                                                 ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
                   "mxgg_peer_barrier")

    def start_dispatch(self, plan: FusedPlan, a_q: Tensor, a_s: Tensor) -> None:
        """Start pushing this rank's rows into their hosts' receive buffers
        (copy engines, one stream per peer); `finish_dispatch` joins them."""
        import ctypes
        from . import _lib
        lib = _lib.load()
        K = a_q.shape[1]
        if K > self.max_k:
            raise ValueError(f"K={K} exceeds the buffers' {self.max_k}")
        a_q = a_q.contiguous()
        a_s = a_s.contiguous()
        cur = torch.cuda.current_stream()
        ready = cur.record_event()
        self._pending = []
        for (d, dst_row, src_row, rows) in plan.copies:
            st = self._streams[d]
            st.wait_event(ready)
            sp = ctypes.c_void_p(st.cuda_stream)
            _lib.check(lib.mxgg_copy_async(ctypes.c_void_p(self.recv_a.ptrs[d] + dst_row * K),
                                           ctypes.c_void_p(a_q.data_ptr() + src_row * K), rows * K, sp),
                       "mxgg_copy_async")
            _lib.check(lib.mxgg_copy_async(ctypes.c_void_p(self.recv_s.ptrs[d] + dst_row * (K // 32)),
                                           ctypes.c_void_p(a_s.data_ptr() + src_row * (K // 32)), rows * (K // 32),
                                           sp), "mxgg_copy_async")
            self._pending.append(st.record_event())
            # the caching allocator must not hand the sources out before the copies finish
            a_q.record_stream(st)
            a_s.record_stream(st)

    def finish_dispatch(self) -> None:
        """The current stream waits for this rank's copies, then for every
        rank's (cross-GPU barrier): the receive buffers are complete."""
        cur = torch.cuda.current_stream()
        for ev in self._pending:
            cur.wait_event(ev)
        self._pending = []
        self.barrier()

    def dispatch(self, plan: FusedPlan, a_q: Tensor, a_s: Tensor) -> None:
        self.start_dispatch(plan, a_q, a_s)
        self.finish_dispatch()

    def self_rows(self, plan: FusedPlan, a_q: Tensor, a_s: Tensor):
        """The rows this rank routed to its own experts (views, no copy)."""
        r0, n = plan.self_row, plan.self_rows
        return a_q[r0:r0 + n], a_s[r0:r0 + n]

    def received(self, plan: FusedPlan, K: int):
        """The peers' dispatched rows as (rows_recv, K) e4m3 and (rows_recv, K/32) scale views."""
        R = plan.rows_recv
        return (self.recv_a.view((R, K), torch.uint8).view(torch.float8_e4m3fn),
                self.recv_s.view((R, K // 32), torch.uint8))

    def gemm(self, plan: FusedPlan, part: str, K: int, w_q: Tensor, w_s: Tensor,
             out_dtype: torch.dtype = torch.bfloat16, a: Optional[tuple] = None) -> None:
        """One part of the expert GEMM with its outputs sent to their owners.

        part "self": the rows this rank routed to itself (`a` = their
        (a_q, a_s), from `self_rows`, or an earlier GEMM's output over them);
        part "remote": the received rows (`a` defaults to the receive buffers)."""
        import ctypes
        from . import _lib
        from .ops import _OUT_DTYPES, _workspace, as_u8, b_format_of
        lib = _lib.load()
        L, N, _ = w_q.shape
        if N > self.max_n:
            raise ValueError(f"N={N} exceeds the output buffer's {self.max_n}")
        seg = plan.self_seg if part == "self" else plan.remote_seg
        R = plan.self_rows if part == "self" else plan.rows_recv
        if a is None:
            if part == "self":
                raise ValueError("the self part needs its rows")
            a = self.received(plan, K)
        a_q, a_s = a[0].contiguous(), as_u8(a[1]).contiguous()
        if a_q.shape[0] != R or a_s.shape != (R, K // 32):
            raise ValueError(f"rows {tuple(a_q.shape)} do not match the plan's ({R}, {K})")
        if R == 0:
            return
        S = seg.offs.numel()
        ws = _workspace(lib.mxgg_grouped_mm_segments_workspace_size(R, N, K, S, L), w_q.device)
        outs = (ctypes.c_void_p * self.world)(*self.out.ptrs)
        rows = (ctypes.c_int64 * self.world)(*plan.dst_rows)
        inboxes = (ctypes.c_void_p * self.world)(*self.inbox.ptrs) if plan.inbox_ok else None
        w_q = w_q.contiguous()
        w_s = as_u8(w_s).contiguous()
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        _lib.check(lib.mxgg_grouped_mm_ep(p(a_q), p(w_q), p(a_s), p(w_s), p(seg.offs), p(seg.expert),
                                          p(seg.dst), p(seg.dst_row), R, N, K, S, L, b_format_of(w_q),
                                          outs, rows, inboxes, self.world, self.rank, _OUT_DTYPES[out_dtype],
                                          p(ws), ws.numel(), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
                   "mxgg_grouped_mm_ep")

    def finish(self, plan: FusedPlan, N: int, out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
        """Barrier (every rank's stores are in), unpack this rank's inbox;
        returns its (rows_local, N) output view."""
        import ctypes
        from . import _lib
        self.barrier()
        es = torch.empty((), dtype=out_dtype).element_size()
        if plan.inbox_ok and plan.remote_blocks.numel() and (N * es) % 64 == 0:
            _lib.check(_lib.load().mxgg_inbox_unpack(ctypes.c_void_p(self.inbox.ptrs[self.rank]),
                                                     ctypes.c_void_p(self.out.ptrs[self.rank]),
                                                     ctypes.c_void_p(plan.remote_blocks.data_ptr()),
                                                     plan.remote_blocks.numel(), N * es,
                                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
                       "mxgg_inbox_unpack")
        return self.out.view((plan.rows_local, N), out_dtype)

    def grouped_mm(self, plan: FusedPlan, a_q: Tensor, a_s: Tensor, w_q: Tensor, w_s: Tensor,
                   out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
        """Fused forward / dgrad: returns (rows_local, N) in this rank's row order."""
        K = a_q.shape[1]
        Kw = w_q.shape[2] * (2 if w_q.dtype == torch.float4_e2m1fn_x2 else 1)
        if Kw != K:
            raise AssertionError(f"K mismatch: activations {K}, weights {Kw}")
        self.start_dispatch(plan, a_q, a_s)
        self.gemm(plan, "self", K, w_q, w_s, out_dtype, a=self.self_rows(plan, a_q, a_s))
        self.finish_dispatch()
        self.gemm(plan, "remote", K, w_q, w_s, out_dtype)
        return self.finish(plan, w_q.shape[1], out_dtype)
