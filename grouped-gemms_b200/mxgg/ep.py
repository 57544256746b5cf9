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
over the replica group: in place over peer memory (``ReplicaSum``), or with
an NCCL all-reduce (``replica_allreduce``).

Nothing here synchronises the device except ``plan_dispatch``, which needs the
received counts on the host to size the NCCL transfers.
"""

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

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
    from .ops import grouped_mm_segments
    recv_q, recv_s = dispatch(plan, a_q, a_s, group=group)
    y = grouped_mm_segments(recv_q, w_q, recv_s, w_s, plan.seg_offs, plan.seg_expert, out_dtype)
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


def wgrad_split_rows(L: int, N: int, K: int, pairs: int) -> Optional[int]:
    """Where a one-expert (L == 1) weight gradient of N x K is cut along N
    into two launches whose parts overlap the replica sum, or None.

    The two launches must not take more rounds of 256 x 256 tiles over
    `pairs` CTA pairs than one launch would (a cut that adds a round costs
    more than the overlap saves), and the grid must hold at least four
    rounds.  Among the cuts that qualify, the one nearest the middle; the
    cut is a multiple of 256 rows, so both parts are whole tiles of the
    one-launch grid."""
    if L != 1 or pairs < 1:
        return None
    nt, kt = -(-N // 256), -(-K // 256)
    if nt < 2 or nt * kt < 4 * pairs:
        return None
    rounds = -(-nt * kt // pairs)
    best = None
    for a in range(1, nt):
        if -(-a * kt // pairs) + -(-(nt - a) * kt // pairs) <= rounds:
            if best is None or abs(2 * a - nt) < abs(2 * best - nt):
                best = a
    return None if best is None else 256 * best


class ReplicaSum:
    """Sums replicated experts' weight gradients over NVLink peer memory, in
    place: the fused counterpart of `replica_allreduce`.

    Collective to construct (every rank allocates `max_bytes` that its peers
    map).  Per step, on every rank:

        g = rs.buffer((L, N, K), torch.bfloat16)     # this rank's replica
        mxgg.ops.wgrad_into(..., out=g)              # write the gradient there
        rs.sum_(placement, g)                        # collective over all ranks

    `sum_` runs a cross-GPU barrier over each replica group, then every
    replica sums its 1/R share of the array from all R replicas (fp32, in
    replica order, one rounding) and stores the result into all of them, then
    a second barrier: each rank's NVLink traffic is 2 (R-1)/R of the array,
    as for a ring all-reduce, but in one kernel at copy speed.  All replicas
    end with identical bits; for R = 2 they equal NCCL's bf16 / fp32 sum.
    The waits are bounded (status bit 64 on timeout, raised by
    `check_status` of a `FusedExpertParallel` or `mxgg.device_status`)."""

    def __init__(self, max_bytes: int, group=None):
        from .peer import PeerBuffer
        dist = _dist()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("the peer-memory replica sum reaches at most 8 ranks (one NVLink domain)")
        self.max_bytes = int(max_bytes)
        self.buf = PeerBuffer(max(self.max_bytes, 256), group)
        self.flags = PeerBuffer(256, group)
        self.epoch = 0
        self._side = torch.cuda.Stream()
        self._pairs = max(1, torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count // 2)

    def close(self) -> None:
        self.buf.close()
        self.flags.close()

    def buffer(self, shape, dtype: torch.dtype) -> Tensor:
        """This rank's replica buffer as a tensor (valid until the next `buffer` use)."""
        return self.buf.view(shape, dtype)

    def sum_(self, placement: ExpertPlacement, t: Tensor) -> Tensor:
        """Collective: every replica of this rank's experts gets the sum of
        all replicas' `t` (no-op without replicas).  A tensor inside this
        rank's buffer (`buffer`, or a part of it) is summed where it lies;
        any other contiguous tensor is copied in and out."""
        import ctypes
        from . import _lib
        from .ops import _OUT_DTYPES
        if placement.world != self.world:
            raise ValueError("placement and process group disagree on the world size")
        if placement.replicas == 1:
            return t
        if t.dtype not in _OUT_DTYPES or not t.is_contiguous():
            raise ValueError("sum_ takes a contiguous bf16, fp16 or fp32 tensor")
        nbytes = t.numel() * t.element_size()
        if nbytes > self.max_bytes:
            raise ValueError(f"{nbytes} bytes exceed the {self.max_bytes}-byte replica buffers")
        # a tensor inside this rank's buffer is summed where it lies (at the
        # same offset in every replica); any other is copied in and out
        off = t.data_ptr() - self.buf.ptrs[self.rank]
        inplace = 0 <= off and off + nbytes <= self.max_bytes and off % 16 == 0
        if not inplace:
            off = 0
            self.buffer(t.shape, t.dtype).copy_(t)
        ranks = placement.replica_group(self.rank)
        me = ranks.index(self.rank)
        lib = _lib.load()
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        flags = (ctypes.c_void_p * len(ranks))(*[self.flags.ptrs[r] for r in ranks])
        bufs = (ctypes.c_void_p * len(ranks))(*[self.buf.ptrs[r] + off for r in ranks])
        # every rank takes the same epochs in the same order (each sum_ is collective)
        self.epoch += 1
        _lib.check(lib.mxgg_peer_barrier(flags, len(ranks), me, self.epoch, stream), "mxgg_peer_barrier")
        _lib.check(lib.mxgg_replica_sum(bufs, len(ranks), me, t.numel(), _OUT_DTYPES[t.dtype], stream),
                   "mxgg_replica_sum")
        self.epoch += 1
        _lib.check(lib.mxgg_peer_barrier(flags, len(ranks), me, self.epoch, stream), "mxgg_peer_barrier")
        if not inplace:
            t.copy_(self.buffer(t.shape, t.dtype))
        return t

    def split_rows(self, L: int, N: int, K: int) -> Optional[int]:
        """Where `wgrad_sum` cuts a one-expert gradient along N, or None
        (`wgrad_split_rows` over this GPU's CTA pairs)."""
        return wgrad_split_rows(L, N, K, self._pairs)

    def wgrad_sum(self, placement: ExpertPlacement, go_t: Tensor, go_scale: Tensor, ia_t: Tensor,
                  ia_scale: Tensor, offs: Tensor, cfg=None, out_dtype: torch.dtype = torch.bfloat16,
                  gemm_done: Optional["torch.cuda.Event"] = None) -> Tensor:
        """Collective: this rank's weight gradient (`mxgg.ops.wgrad_into`,
        row-major scales) written into its replica buffer and summed over the
        replicas; returns the (L, N, K) buffer view.

        With one local expert, no tuned config and a large enough grid
        (`split_rows`), the gradient is computed in two launches cut along N,
        and the first part's replica sum runs on a side stream while the
        second part computes: the sum's NVLink traffic overlaps the GEMM.
        Each part is whole tiles of the same grid, so the bits are those of
        one launch.  `gemm_done`, if given, is recorded on the current stream
        after the last GEMM launch (for timing the phases)."""
        from .ops import wgrad_into
        L, N, K = offs.shape[0], go_t.shape[0], ia_t.shape[0]
        out = self.buffer((L, N, K), out_dtype)
        cut = self.split_rows(L, N, K) if placement.replicas > 1 and cfg is None else None
        if cut is None:
            wgrad_into(go_t, go_scale, ia_t, ia_scale, offs, out, cfg)
            if gemm_done is not None:
                gemm_done.record()
            return self.sum_(placement, out)
        flat = out.view(N, K)
        first, second = flat[:cut].view(1, cut, K), flat[cut:].view(1, N - cut, K)
        wgrad_into(go_t[:cut], go_scale[:cut], ia_t, ia_scale, offs, first)
        cur = torch.cuda.current_stream()
        self._side.wait_stream(cur)
        with torch.cuda.stream(self._side):
            self.sum_(placement, first)
        wgrad_into(go_t[cut:], go_scale[cut:], ia_t, ia_scale, offs, second)
        if gemm_done is not None:
            gemm_done.record()
        # every rank's second sum starts after its first: the barriers' epochs stay in order
        cur.wait_stream(self._side)
        self.sum_(placement, second)
        return out


# ----------------------------------------------------------------------------
# Fused path: peer-memory dispatch, combine fused into the GEMM epilogue.
# ----------------------------------------------------------------------------
@dataclass
class _Segments:
    offs: Tensor                 # int32 cumulative ends of the segments (rows of the A operand)
    expert: Tensor               # local expert of each segment
    dst: Tensor                  # output destination of each segment's rows
    dst_row: Tensor              # first row of the segment there
    src: Tensor                  # source id of each segment's rows: rank + world * piece


@dataclass
class FusedPlan:
    """Routing of one fused expert-parallel call, as seen by one rank.

    Receive layout of rank d (its A operand): sources in arrival order d,
    d-1, d-2, ..., each source's rows grouped by local expert.  Its own rows
    keep their slot but are read in place from the caller's tensor.  Rank s
    sends to s+1, s+2, ... in turn, so every receiver gets its sources one
    after another in that order."""

    rows_local: int
    rows_recv: int               # all rows this rank multiplies (its own included)
    copies: List[tuple]          # (dest rank, first row there, first local row, rows, flag slot there) to
                                 #  peers, in sending order
    pack: List[tuple]            # (dest rank, cumulative segment ends (device), first 128-row scale slab
                                 #  there, first local row, rows), this rank included
    self_base: int               # local row of the first row this rank routes to itself
    seg: _Segments               # world * L segments over the receive buffer
    local_seg: _Segments         # the same segments with every row kept here, in receive order
    dst_rows: List[int]          # local rows of every rank (the output buffers' heights)
    inbox_ok: bool               # every segment starts on a 32-row boundary: peers' blocks go by inbox
    remote_blocks: Tensor        # this rank's 32-row blocks computed by peers (unpacked from its inbox)


MAX_SOURCE_IDS = 32          # source-flag slots the GEMM tracks (a 32-bit readiness mask)
MAX_SEGMENTS = 256           # segments the GEMM's in-kernel group table holds
PIECE_ALIGN = 256            # rows: a piece cut lands on the GEMM's tile grid of its segment
MAX_PIECES = 4               # pieces per (source, destination) block


def _piece_cuts(seg_rows: List[int], n_pieces: int, align: int = PIECE_ALIGN) -> List[int]:
    """Row offsets inside one source's block (ascending, neither 0 nor the
    block's end) that cut it into about `n_pieces` equal pieces.  Each cut
    is moved forward to a segment start or to a multiple of `align` rows
    past one, so that no tile of the GEMM straddles two pieces and the
    128-row scale slabs of the cut segments are those of the uncut ones."""
    total = sum(seg_rows)
    cuts: List[int] = []
    for c in range(1, n_pieces):
        t = (c * total) // n_pieces
        lo, cut = 0, total
        for r in seg_rows:
            if t < lo + r:
                cut = lo + min(-(-(t - lo) // align) * align, r)
                break
            lo += r
        if 0 < cut < total and (not cuts or cut > cuts[-1]):
            cuts.append(cut)
    return cuts


def fused_layout(C: List[List[int]], pl: ExpertPlacement, rank: int, piece_rows: int = 2048) -> dict:
    """The fused path's routing arithmetic for `rank`, from every rank's
    per-expert row counts C[s][e] (rows sorted by expert on each rank).

    Receiver d's layout: sources in arrival order d, d-1, d-2, ..., each
    source's rows grouped by d's local experts.  A peer's block of rows
    travels in up to MAX_PIECES pieces of at least `piece_rows` rows (0: one
    piece), each copied and flagged on its own, so the GEMM starts on a
    piece as soon as it lands instead of waiting for the whole block; the
    segments are cut at the pieces' edges and carry the piece's source id
    s + world * piece (flag slot of that id).  Returns plain lists:
      copies   (dest, first row there, first local row, rows, flag slot there), to peers, in sending
               order d+1, d+2, ...
      pack     (dest, cumulative segment ends, first 128-row scale slab there, first local row, rows),
               this rank included
      seg      offs / expert / src / dst / dst_row / local_row of this rank's receive segments
      self_base, rows_recv, rows_local, dst_rows, need_recv, inbox_ok, remote_blocks
    """
    world, E = pl.world, pl.n_experts
    max_pieces = min(MAX_PIECES, MAX_SOURCE_IDS // world)
    if piece_rows <= 0 or world * pl.local + world * (max_pieces - 1) > MAX_SEGMENTS:
        max_pieces = 1

    def n_pieces(rows):
        return max(1, min(max_pieces, rows // piece_rows)) if max_pieces > 1 else 1

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

    def order(d):                       # sources, in arrival order
        return [(d - j) % world for j in range(world)]

    def seg_rows(s, d):
        return [C[s][e] if pl.dest(s, e) == d else 0 for e in pl.experts_of(d)]

    # where each source's rows and scale slabs start at each receiver
    recv_off = [[0] * world for _ in range(world)]
    m0 = [[0] * world for _ in range(world)]
    for d in range(world):
        r = m = 0
        for s in order(d):
            recv_off[s][d], m0[s][d] = r, m
            r += send[s][d]
            m += sum((c + 127) // 128 for c in seg_rows(s, d))   # 128-row scale slabs
    copies, pack = [], []
    for j in range(world):
        d = (rank + j) % world
        if send[rank][d]:
            if d != rank:
                b = [0] + _piece_cuts(seg_rows(rank, d), n_pieces(send[rank][d])) + [send[rank][d]]
                for c in range(len(b) - 1):
                    copies.append((d, recv_off[rank][d] + b[c], start[rank][d] + b[c], b[c + 1] - b[c],
                                   rank + world * c))
            cum, acc = [], 0
            for c in seg_rows(rank, d):
                acc += c
                cum.append(acc)
            pack.append((d, cum, m0[rank][d], start[rank][d], send[rank][d]))
    seg = {"offs": [], "expert": [], "src": [], "dst": [], "dst_row": [], "local_row": []}
    total = 0
    for s in order(rank):
        rows_s = seg_rows(s, rank)
        # own rows are read in place and never wait: one piece
        cuts = [] if s == rank else _piece_cuts(rows_s, n_pieces(send[s][rank]))
        pos = 0                         # row inside the source's block
        for le, (e, rows) in enumerate(zip(pl.experts_of(rank), rows_s)):
            edges = [pos] + [c for c in cuts if pos < c < pos + rows] + [pos + rows]
            for a, b in zip(edges[:-1], edges[1:]):
                piece = sum(1 for c in cuts if c <= a)
                seg["local_row"].append(total)
                total += b - a
                seg["offs"].append(total)
                seg["expert"].append(le)
                seg["src"].append(s + world * piece)
                seg["dst"].append(s)
                seg["dst_row"].append(sum(C[s][:e]) + a - pos)
            pos += rows
    blocks, row = [], 0
    for e in range(E):
        if pl.dest(rank, e) != rank:
            blocks.extend(range(row // 32, (row + C[rank][e]) // 32))
        row += C[rank][e]
    return {"copies": copies, "pack": pack, "seg": seg, "self_base": start[rank][rank] - recv_off[rank][rank],
            "rows_recv": total, "rows_local": sum(C[rank]), "dst_rows": [sum(C[d]) for d in range(world)],
            "need_recv": [sum(send[s][d] for s in range(world)) for d in range(world)],
            "inbox_ok": all(c % 32 == 0 for row_ in C for c in row_), "remote_blocks": blocks}


class FusedExpertParallel:
    """Expert-parallel forward / dgrad over NVLink peer memory, with the
    dispatch streamed into the GEMM and the combine fused into its epilogue.

    Collective to construct (it allocates and maps the shared buffers).  Per
    call (`grouped_mm`):

    1. each rank packs the scale atoms of its rows straight into every
       destination's atom buffer (in the destination's tile numbering), then,
       on a side stream, copies its rows into the destinations' receive
       buffers one destination after another (copy engine), a large block in
       up to four pieces, and after each copy raises that piece's flag there;
    2. meanwhile the GEMM runs over the whole receive buffer: its producer
       loads a segment's tiles as soon as the segment's piece has raised its
       flag (a bounded wait), and its epilogue sends every output block to the
       rank that owns the rows (TMA stores for its own rows; 2 KB bulk copies
       into the owner's inbox for peers'), so both transfers overlap the math;
    3. a cross-GPU barrier, then each rank unpacks its inbox into its output.

    The returned tensor is a view of this rank's shared output buffer: use it
    before the next call.
    """

    def __init__(self, placement: ExpertPlacement, max_recv_rows: int, max_local_rows: int, max_k: int, max_n: int,
                 group=None):
        from . import _lib
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
        lib = _lib.load()
        self.recv_a = PeerBuffer(max(self.max_recv_rows * self.max_k, 256), group)
        self.atoms = PeerBuffer(max(lib.mxgg_ep_atom_bytes(self.max_recv_rows, self.max_k, 256), 256), group)
        self.out = PeerBuffer(max(self.max_local_rows * self.max_n * 4, 256), group)
        self.inbox = PeerBuffer(max(self.max_local_rows * self.max_n * 4, 256), group)
        self.flags = PeerBuffer(256, group)          # barrier slots
        self.src_flags = PeerBuffer(4 * MAX_SOURCE_IDS, group)   # streaming-dispatch slots, one per source id
        self.epoch = 0
        self.src_epoch = 0
        self._side = torch.cuda.Stream()
        self._side_pending = False
        self._a_self = None
        # every rank's capacities, so a plan that overflows any of them fails on all ranks alike
        caps = [None] * self.world
        dist.all_gather_object(caps, (self.max_recv_rows, self.max_local_rows), group=group)
        self._caps = caps

    def close(self) -> None:
        for b in (self.recv_a, self.atoms, self.out, self.inbox, self.flags, self.src_flags):
            b.close()

    # -------------------------------------------------------------- planning
    def plan(self, expert_counts: Sequence[int], placement: Optional[ExpertPlacement] = None,
             piece_rows: int = 2048) -> FusedPlan:
        """Collective: all-gather every rank's per-expert counts and derive the
        copies, atom packing, segment tables and output heights.  The shared
        buffers do not depend on the placement, so one instance serves several
        (`placement` overrides the constructor's for this plan).  A peer's
        block of at least 2 * `piece_rows` rows travels in pieces that the GEMM
        starts on one by one (`fused_layout`); every rank must pass the same
        value.

        It also gathers every rank's device status word (read and cleared
        here) and raises MxggError on all ranks alike when any of them is set:
        the previous call's output must then be discarded.  Callers that reuse
        one plan for many calls check with `check_status` instead."""
        from . import _lib
        dist = _dist()
        pl, world, rank = placement or self.placement, self.world, self.rank
        if pl.world != world:
            raise ValueError("placement and process group disagree on the world size")
        E = pl.n_experts
        dev = torch.device("cuda", torch.cuda.current_device())
        counts = [int(c) for c in expert_counts]
        if len(counts) != E or any(c < 0 for c in counts):
            raise ValueError("expert_counts must hold E non-negative counts")
        # The previous call's device-side error word travels with the counts:
        # a bounded cross-GPU wait that gave up (a peer's rows or barrier
        # slot never arrived: status bits 64 / 128) left stale rows in that
        # call's output, and every rank raises here together, before the next
        # collective, instead of carrying on with wrong numbers.
        status = _lib.device_status(clear=True, stream=torch.cuda.current_stream().cuda_stream)
        mine = torch.tensor(counts + [status], dtype=torch.int64, device=dev)
        allc = torch.empty(world, E + 1, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(allc, mine, group=self.group)
        gathered = allc.tolist()                              # one device sync
        bad = {r: row[E] for r, row in enumerate(gathered) if row[E] != 0}
        if bad:
            raise _lib.MxggError("fused expert parallelism: a device-side wait gave up in the previous call "
                                 "(rank: status word) " + ", ".join(f"{r}: {v:#x}" for r, v in sorted(bad.items())))
        C = [row[:E] for row in gathered]                     # C[s][e]
        lay = fused_layout(C, pl, rank, piece_rows)
        for d in range(world):
            if lay["need_recv"][d] > self._caps[d][0] or lay["dst_rows"][d] > self._caps[d][1]:
                raise ValueError(f"fused EP buffers of rank {d} too small: {lay['need_recv'][d]} received / "
                                 f"{lay['dst_rows'][d]} local rows for {self._caps[d][0]} / {self._caps[d][1]}")
        i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)  # noqa: E731
        pack = [(d, i32(cum), m0, src_row, rows) for (d, cum, m0, src_row, rows) in lay["pack"]]
        seg = lay["seg"]
        o, x, sr = i32(seg["offs"]), i32(seg["expert"]), i32(seg["src"])
        return FusedPlan(rows_local=lay["rows_local"], rows_recv=lay["rows_recv"], copies=lay["copies"], pack=pack,
                         self_base=lay["self_base"],
                         seg=_Segments(o, x, i32(seg["dst"]), i32(seg["dst_row"]), sr),
                         local_seg=_Segments(o, x, i32([rank] * len(seg["offs"])), i32(seg["local_row"]), sr),
                         dst_rows=lay["dst_rows"], inbox_ok=lay["inbox_ok"],
                         remote_blocks=i32(lay["remote_blocks"] if lay["inbox_ok"] else []))

    def check_status(self) -> None:
        """Collective: raise MxggError on every rank when any rank's device
        status word is set (a bounded cross-GPU wait gave up in an earlier
        call, so that call's output holds stale rows).  Reads and clears the
        word; one small all-gather and a device sync."""
        from . import _lib
        dist = _dist()
        st = _lib.device_status(clear=True, stream=torch.cuda.current_stream().cuda_stream)
        dev = torch.device("cuda", torch.cuda.current_device())
        allst = torch.empty(self.world, dtype=torch.int64, device=dev)
        dist.all_gather_into_tensor(allst, torch.tensor([st], dtype=torch.int64, device=dev), group=self.group)
        bad = {r: v for r, v in enumerate(allst.tolist()) if v != 0}
        if bad:
            raise _lib.MxggError("fused expert parallelism: a device-side wait gave up "
                                 "(rank: status word) " + ", ".join(f"{r}: {v:#x}" for r, v in sorted(bad.items())))

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

    def dispatch(self, plan: FusedPlan, a_q: Tensor, a_s: Tensor) -> None:
        """Start the streamed dispatch of this rank's rows (sorted by expert):
        scale atoms into every destination's atom buffer (on the current
        stream), then row copies and per-destination flags (side stream)."""
        import ctypes
        from . import _lib
        lib = _lib.load()
        K = a_q.shape[1]
        if K > self.max_k:
            raise ValueError(f"K={K} exceeds the buffers' {self.max_k}")
        a_q = a_q.contiguous()
        a_s = a_s.contiguous()
        self.src_epoch += 1
        cur = torch.cuda.current_stream()
        sp = ctypes.c_void_p(cur.cuda_stream)
        atom_bytes_per_slab = (K + 127) // 128 * 512
        n = len(plan.pack)
        if n:
            # every destination's atoms in one launch
            i64 = ctypes.c_int64 * n
            _lib.check(lib.mxgg_pack_a_atoms_multi(
                ctypes.c_void_p(a_s.data_ptr()), K, n, i64(*[src_row for (_, _, _, src_row, _) in plan.pack]),
                i64(*[rows for (_, _, _, _, rows) in plan.pack]),
                (ctypes.c_void_p * n)(*[cum.data_ptr() for (_, cum, _, _, _) in plan.pack]),
                i64(*[cum.numel() for (_, cum, _, _, _) in plan.pack]),
                (ctypes.c_void_p * n)(*[self.atoms.ptrs[d] + m0 * atom_bytes_per_slab
                                        for (d, _, m0, _, _) in plan.pack]), sp),
                "mxgg_pack_a_atoms_multi")
        side = self._side
        side.wait_stream(cur)
        ssp = ctypes.c_void_p(side.cuda_stream)
        for (d, dst_row, src_row, rows, slot) in plan.copies:
            _lib.check(lib.mxgg_copy_async(ctypes.c_void_p(self.recv_a.ptrs[d] + dst_row * K),
                                           ctypes.c_void_p(a_q.data_ptr() + src_row * K), rows * K, ssp),
                       "mxgg_copy_async")
            _lib.check(lib.mxgg_peer_signal(ctypes.c_void_p(self.src_flags.ptrs[d] + 4 * slot),
                                            self.src_epoch, ssp), "mxgg_peer_signal")
        # (a destination this rank sends no rows to never waits for it: its segments are empty)
        a_q.record_stream(side)
        a_s.record_stream(side)
        self._side_pending = True
        self._a_self = (a_q, plan.self_base)     # this rank's own rows, read in place by gemm_received

    def received(self, plan: FusedPlan, K: int) -> Tensor:
        """The receive buffer as (rows_recv, K) e4m3 (complete after `finish`)."""
        return self.recv_a.view((plan.rows_recv, K), torch.uint8).view(torch.float8_e4m3fn)

    def _ep_gemm(self, plan, seg, a_q, K, w_q, w_s, out_dtype, outs, rows, inboxes, a_atoms, src_flags, a_s=None,
                 a_self=None, quant=None):
        import ctypes
        from . import _lib
        from .ops import _OUT_DTYPES, _workspace, as_u8, b_format_of
        lib = _lib.load()
        L, N, _ = w_q.shape
        R = a_q.shape[0]
        if R == 0:
            return
        S = seg.offs.numel()
        ws = _workspace(lib.mxgg_grouped_mm_segments_workspace_size(R, N, K, S, L), w_q.device)
        w_q = w_q.contiguous()
        w_s = as_u8(w_s).contiguous()
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        scale = p(as_u8(a_s).contiguous()) if a_s is not None else ctypes.c_void_p(a_atoms)
        _lib.check(lib.mxgg_grouped_mm_ep(p(a_q), p(w_q), scale, p(w_s), p(seg.offs), p(seg.expert), p(seg.dst),
                                          p(seg.dst_row), R, N, K, S, L, b_format_of(w_q), outs, rows, inboxes,
                                          self.world, self.rank,
                                          ctypes.c_void_p(a_atoms) if a_atoms else None,
                                          ctypes.c_void_p(src_flags) if src_flags else None, self.src_epoch,
                                          p(seg.src), p(a_self[0]) if a_self else None, a_self[0].shape[0] if a_self else 0,
                                          self.rank, a_self[1] if a_self else 0,
                                          p(quant[0]) if quant else None, p(quant[1]) if quant else None,
                                          _OUT_DTYPES[out_dtype], p(ws), ws.numel(),
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)),
                   "mxgg_grouped_mm_ep")

    def gemm_received(self, plan: FusedPlan, K: int, w_q: Tensor, w_s: Tensor,
                      out_dtype: torch.dtype = torch.bfloat16, local_out: Optional[Tensor] = None,
                      local_mx: Optional[Tuple[Tensor, Tensor]] = None) -> None:
        """GEMM over the receive buffer as it fills (after `dispatch`).  Output
        rows go to their owners, or, with `local_out` ((rows_recv, N)), stay
        here in receive order.  `local_mx` = (data (rows_recv, N) e4m3, scales
        (rows_recv, N//32) uint8): the rows stay here and are written in MXFP8
        by the epilogue (to_mx of the out_dtype output, fused); `local_out`
        may then be None."""
        import ctypes
        L, N, _ = w_q.shape
        if N > self.max_n:
            raise ValueError(f"N={N} exceeds the output buffer's {self.max_n}")
        a = self.recv_a.view((plan.rows_recv, K), torch.uint8)
        if local_out is not None or local_mx is not None:
            if local_out is not None and (local_out.shape != (plan.rows_recv, N) or not local_out.is_contiguous()):
                raise ValueError("local_out must be a contiguous (rows_recv, N) tensor")
            if local_mx is not None and (local_mx[0].shape != (plan.rows_recv, N) or
                                         local_mx[1].shape != (plan.rows_recv, N // 32) or
                                         not (local_mx[0].is_contiguous() and local_mx[1].is_contiguous())):
                raise ValueError("local_mx must be contiguous (rows_recv, N) data and (rows_recv, N//32) scales")
            here = local_out.data_ptr() if local_out is not None else 0
            outs = (ctypes.c_void_p * self.world)(*[here if r == self.rank else 0 for r in range(self.world)])
            rows = (ctypes.c_int64 * self.world)(*[plan.rows_recv if r == self.rank else 0
                                                   for r in range(self.world)])
            self._ep_gemm(plan, plan.local_seg, a, K, w_q, w_s, out_dtype, outs, rows, None,
                          self.atoms.ptrs[self.rank], self.src_flags.ptrs[self.rank], a_self=self._a_self,
                          quant=local_mx)
            return
        outs = (ctypes.c_void_p * self.world)(*self.out.ptrs)
        rows = (ctypes.c_int64 * self.world)(*plan.dst_rows)
        inboxes = (ctypes.c_void_p * self.world)(*self.inbox.ptrs) if plan.inbox_ok else None
        self._ep_gemm(plan, plan.seg, a, K, w_q, w_s, out_dtype, outs, rows, inboxes,
                      self.atoms.ptrs[self.rank], self.src_flags.ptrs[self.rank], a_self=self._a_self)

    def gemm_local(self, plan: FusedPlan, a_q: Tensor, a_s: Tensor, w_q: Tensor, w_s: Tensor,
                   out_dtype: torch.dtype = torch.bfloat16) -> None:
        """GEMM over local rows laid out like the receive buffer (for example
        the quantised output of `gemm_received(local_out=...)`), output rows
        to their owners."""
        import ctypes
        K = a_q.shape[1]
        if a_q.shape[0] != plan.rows_recv:
            raise ValueError("local rows must match the plan's receive layout")
        outs = (ctypes.c_void_p * self.world)(*self.out.ptrs)
        rows = (ctypes.c_int64 * self.world)(*plan.dst_rows)
        inboxes = (ctypes.c_void_p * self.world)(*self.inbox.ptrs) if plan.inbox_ok else None
        self._ep_gemm(plan, plan.seg, a_q.contiguous(), K, w_q, w_s, out_dtype, outs, rows, inboxes, None, None,
                      a_s=a_s)

    def finish(self, plan: FusedPlan, N: int, out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
        """Join the copies, barrier (every rank's stores are in), unpack this
        rank's inbox; returns its (rows_local, N) output view."""
        import ctypes
        from . import _lib
        if self._side_pending:
            torch.cuda.current_stream().wait_stream(self._side)
            self._side_pending = False
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
        self.dispatch(plan, a_q, a_s)
        self.gemm_received(plan, K, w_q, w_s, out_dtype)
        return self.finish(plan, w_q.shape[1], out_dtype)
