"""Grouped GEMMs on operands that live in pinned host memory, with the
host <-> device copies overlapped with the math.

Called one after another, the three steps of such a call (copy the operands
in, run the GEMM, copy the result out) leave the GPU idle for most of the
call: over PCIe the copies take several times longer than the GEMM.  Here a
call is cut into pieces that run on three streams, so that piece c's GEMM
overlaps piece c+1's copy in and piece c-1's copy out:

* forward / dgrad (``grouped_mm``): with several experts, a piece is a run of
  consecutive groups together with their experts' weights, so the weights
  arrive piece by piece too; with one expert, the weights go first and a
  piece is a run of rows;
* wgrad (``wgrad``): the activations (``ia_t``, the right operand) go first
  and a piece is a run of 256 rows of ``go_t``, i.e. of every expert's
  gradient rows.

Every piece is an ordinary call of the reference-named entry point
(``kernels.triton_mxfp8_grouped_mm`` / ``kernels.triton_mxfp8_wgrad``) on
device views of the operands.  Under the whole-tile schedule each output
element is the same MMA chain over the whole contraction whichever piece
computes it, so the results are bit-identical to a single call.  (A tuned
table entry may send a wgrad shape to the split-tail schedule, which sums
fp32 partial tiles; pieces then split different tiles and may round some
elements differently.)

The reference has no host-operand path: its callers copy to the device
themselves (``bench.py`` of the reference times device-resident operands).
"""

from typing import List, Optional, Sequence, Tuple

import torch
from torch import Tensor


def _bytes(t: Tensor) -> Tensor:
    return t.contiguous().view(torch.uint8).reshape(-1)


def row_cuts(rows: int, pieces: int, align: int = 256) -> List[int]:
    """Cut points [0, ..., rows] of about `pieces` equal runs of rows, on
    multiples of `align` (fewer runs when `rows` is short)."""
    cuts = [0]
    for c in range(1, pieces):
        x = (c * rows // pieces) // align * align
        if cuts[-1] < x < rows:
            cuts.append(x)
    cuts.append(rows)
    return cuts


def group_pieces(ends: Sequence[int], row_bytes: int, expert_bytes: int,
                 pieces: int) -> List[Tuple[int, int, int, int]]:
    """(first group, end group, first row, end row) of each piece of a
    forward call: with several groups, runs of whole groups of about equal
    bytes to copy in (their rows plus their experts' weights); with one,
    runs of rows."""
    E, M = len(ends), (ends[-1] if ends else 0)
    if E >= 2 and pieces > 1:
        starts = [0] + list(ends[:-1])
        cost = [(ends[g] - starts[g]) * row_bytes + expert_bytes for g in range(E)]
        total, acc, out, g0 = sum(cost), 0, [], 0
        for g in range(E):
            acc += cost[g]
            if acc * pieces >= total * (len(out) + 1) and g + 1 < E and len(out) + 1 < pieces:
                out.append((g0, g + 1, starts[g0], ends[g]))
                g0 = g + 1
        out.append((g0, E, starts[g0], M))
        return out
    cuts = row_cuts(M, pieces)
    return [(0, E, cuts[c], cuts[c + 1]) for c in range(len(cuts) - 1)]


class HostPipeline:
    """Three streams (copy in, compute, copy out) and device staging buffers,
    reused from call to call.  Host tensors must be pinned and contiguous.
    The call is ordered after the work already on the caller's current
    stream, and the current stream waits for its last copy out, so events
    recorded around the call on that stream bracket all of it."""

    def __init__(self, device: Optional[torch.device] = None, pieces: int = 8):
        if pieces < 1:
            raise ValueError("pieces must be >= 1")
        self.device = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.pieces = int(pieces)
        self.h2d = torch.cuda.Stream(self.device)
        self.comp = torch.cuda.Stream(self.device)
        self.d2h = torch.cuda.Stream(self.device)
        self._bufs = {}

    # ------------------------------------------------------------ helpers
    def _buf(self, name: str, like: Tensor) -> Tensor:
        """A device tensor shaped like host tensor `like` (storage reused)."""
        nb = like.numel() * like.element_size()
        b = self._bufs.get(name)
        if b is None or b.numel() < nb:
            b = torch.empty(max(nb, 1), dtype=torch.uint8, device=self.device)
            self._bufs[name] = b
        return b[:nb].view(like.dtype).view(like.shape)

    @staticmethod
    def _check_host(*ts: Tensor) -> None:
        for t in ts:
            if t.is_cuda or not t.is_pinned() or not t.is_contiguous():
                raise ValueError("host operands must be contiguous pinned CPU tensors")

    def _start(self) -> None:
        cur = torch.cuda.current_stream(self.device)
        for s in (self.h2d, self.comp, self.d2h):
            s.wait_stream(cur)

    def _finish(self) -> None:
        torch.cuda.current_stream(self.device).wait_stream(self.d2h)

    def _group_pieces(self, ends: Sequence[int], row_bytes: int, expert_bytes: int) -> List[Tuple[int, int, int, int]]:
        return group_pieces(ends, row_bytes, expert_bytes, self.pieces)

    # ------------------------------------------------------------ calls
    def grouped_mm(self, a: Tensor, b: Tensor, a_scale: Tensor, b_scale: Tensor, group_end_offsets,
                   out: Tensor, out_dtype: torch.dtype = torch.bfloat16) -> Tensor:
        """`kernels.triton_mxfp8_grouped_mm` (forward or dgrad) on host
        operands: a (M, K) e4m3, b (E, N, K), scales row-major, the group end
        offsets as a CPU int tensor or list; the (M, N) result is written
        into the pinned host tensor `out`, which is returned."""
        import kernels
        self._check_host(a, b, a_scale, b_scale, out)
        ends = [int(x) for x in (group_end_offsets.tolist() if torch.is_tensor(group_end_offsets)
                                 else group_end_offsets)]
        M, K = a.shape
        E, N = b.shape[0], b.shape[1]
        if len(ends) != E or (ends and ends[-1] != M) or out.shape != (M, N) or out.dtype != out_dtype:
            raise ValueError("grouped_mm: offsets must end at M and out must be (M, N) of out_dtype")
        pieces = self._group_pieces(ends, a.shape[1] + a_scale.shape[1],
                                    (b.numel() * b.element_size() + b_scale.numel()) // max(E, 1))
        # device views; relative group ends of every piece in one pinned table
        a_d, as_d = self._buf("a", a), self._buf("as", a_scale)
        b_d, bs_d = self._buf("b", b), self._buf("bs", b_scale)
        tab = []
        for (g0, g1, r0, r1) in pieces:
            tab += [min(max(ends[g] - r0, 0), r1 - r0) for g in range(g0, g1)]
        tab_h = torch.tensor(tab or [0], dtype=torch.int32).pin_memory()
        tab_d = self._buf("offs", tab_h)
        self._start()
        h2d_done = []
        with torch.cuda.stream(self.h2d):
            tab_d.copy_(tab_h, non_blocking=True)
            b_all = pieces[0][0] == 0 and pieces[0][1] == E and len(pieces) > 1   # one expert: weights first
            if b_all:
                _bytes(b_d).copy_(_bytes(b), non_blocking=True)
                _bytes(bs_d).copy_(_bytes(b_scale), non_blocking=True)
            for (g0, g1, r0, r1) in pieces:
                if not b_all:
                    b_d[g0:g1].copy_(b[g0:g1], non_blocking=True)
                    bs_d[g0:g1].copy_(b_scale[g0:g1], non_blocking=True)
                if r1 > r0:
                    a_d[r0:r1].copy_(a[r0:r1], non_blocking=True)
                    as_d[r0:r1].copy_(a_scale[r0:r1], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.h2d)
                h2d_done.append(ev)
        off = 0
        for c, (g0, g1, r0, r1) in enumerate(pieces):
            n_g = g1 - g0
            offs = tab_d[off:off + n_g]
            off += n_g
            if r1 == r0:
                continue
            self.comp.wait_event(h2d_done[c])
            with torch.cuda.stream(self.comp):
                y = kernels.triton_mxfp8_grouped_mm(a_d[r0:r1], b_d[g0:g1], as_d[r0:r1], bs_d[g0:g1], offs,
                                                    out_dtype=out_dtype)
                y.record_stream(self.d2h)
            self.d2h.wait_stream(self.comp)
            with torch.cuda.stream(self.d2h):
                out[r0:r1].copy_(y, non_blocking=True)
        self._finish()
        return out

    def wgrad(self, go_t: Tensor, go_scale: Tensor, ia_t: Tensor, ia_scale: Tensor, group_end_offsets,
              out: Tensor) -> Tensor:
        """`kernels.triton_mxfp8_wgrad` on host operands: go_t (N, M), ia_t
        (K, M) e4m3 with row-major (., M/32) scales, the group end offsets as
        a CPU int tensor or list; the (E, N, K) result (bf16 or the dtype of
        `out`) is written into the pinned host tensor `out`."""
        import kernels
        self._check_host(go_t, go_scale, ia_t, ia_scale, out)
        ends = [int(x) for x in (group_end_offsets.tolist() if torch.is_tensor(group_end_offsets)
                                 else group_end_offsets)]
        N, M = go_t.shape
        K = ia_t.shape[0]
        E = len(ends)
        if out.shape != (E, N, K):
            raise ValueError(f"wgrad: out must be ({E}, {N}, {K})")
        cuts = row_cuts(N, self.pieces)
        g_d, gs_d = self._buf("a", go_t), self._buf("as", go_scale)
        x_d, xs_d = self._buf("b", ia_t), self._buf("bs", ia_scale)
        offs_h = torch.tensor(ends, dtype=torch.int32).pin_memory()
        offs_d = self._buf("offs", offs_h)
        self._start()
        h2d_done = []
        with torch.cuda.stream(self.h2d):
            offs_d.copy_(offs_h, non_blocking=True)
            _bytes(x_d).copy_(_bytes(ia_t), non_blocking=True)
            _bytes(xs_d).copy_(_bytes(ia_scale), non_blocking=True)
            for c in range(len(cuts) - 1):
                n0, n1 = cuts[c], cuts[c + 1]
                g_d[n0:n1].copy_(go_t[n0:n1], non_blocking=True)
                gs_d[n0:n1].copy_(go_scale[n0:n1], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.h2d)
                h2d_done.append(ev)
        for c in range(len(cuts) - 1):
            n0, n1 = cuts[c], cuts[c + 1]
            self.comp.wait_event(h2d_done[c])
            with torch.cuda.stream(self.comp):
                y = kernels.triton_mxfp8_wgrad(g_d[n0:n1], gs_d[n0:n1], x_d, xs_d, offs_d, out_dtype=out.dtype)
                y.record_stream(self.d2h)
            self.d2h.wait_stream(self.comp)
            with torch.cuda.stream(self.d2h):
                for e in range(E):
                    out[e, n0:n1].copy_(y[e], non_blocking=True)
        self._finish()
        return out
