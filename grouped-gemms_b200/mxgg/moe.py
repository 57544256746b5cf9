"""Mixture-of-experts layer on the mxgg kernels (forward).

    logits -> top-2 routing -> quantise-on-dispatch (gather + to_mx, one pass)
    -> up projection (d_model -> d_ff) per expert, to_mx fused into its epilogue
    -> down projection (d_ff -> d_model) per expert -> weighted top-2 combine

Expert weights are MXFP8, or MXFP4 (e2m1) with MXFP8 activations.  Each
expert's rows are padded to a multiple of 32 (zero rows), the group alignment
the weight-gradient kernels and the inbox transfers need.  With a
`FusedExpertParallel`, rank r hosts its placement's experts: rows travel to
the hosting rank by peer copies, the up projection reads them in place, and
the down projection stores its tiles straight to the rows' owners.  The
routing and the final weighted sum are small torch ops; the GEMMs and the
quantisers are the sm_100a kernels.
"""

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch
from torch import Tensor

from . import _lib
from .ep import ExpertPlacement, FusedExpertParallel
from .ops import _IN_DTYPES, _ptr, _stream, grouped_mm_mx, grouped_mm_segments, to_mx, to_mx_fp4

PAD = 32


def route_top2(logits: Tensor):
    """Softmax over experts, the two largest, renormalised: (experts (T, 2), weights (T, 2) fp32)."""
    probs = torch.softmax(logits.float(), dim=-1)
    w, e = torch.topk(probs, 2, dim=-1)
    return e, w / w.sum(-1, keepdim=True)


@dataclass
class DispatchLayout:
    row_index: Tensor     # (P,) int32 source token of every padded row, -1 for padding
    counts: list          # (E,) padded rows per expert (multiples of PAD)
    pair_pos: Tensor      # (T, 2) int64 padded row of each (token, choice)


def dispatch_layout(experts: Tensor, n_experts: int, pad: int = PAD) -> DispatchLayout:
    """Rows sorted by expert, every expert's rows padded to a multiple of `pad`."""
    T, k = experts.shape
    flat = experts.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=n_experts)
    padded = (counts + pad - 1) // pad * pad
    start_pad = torch.cumsum(padded, 0) - padded
    start = torch.cumsum(counts, 0) - counts
    e_sorted = flat[order]
    pos_sorted = start_pad[e_sorted] + (torch.arange(flat.numel(), device=flat.device) - start[e_sorted])
    P = int(padded.sum())
    row_index = torch.full((P,), -1, dtype=torch.int32, device=flat.device)
    row_index[pos_sorted] = (order // k).to(torch.int32)
    pair_pos = torch.empty_like(flat)
    pair_pos[order] = pos_sorted
    return DispatchLayout(row_index=row_index, counts=padded.tolist(), pair_pos=pair_pos.reshape(T, k))


def quantize_gather(x: Tensor, row_index: Tensor):
    """(scales, q) of to_mx(x[row_index]) with zero rows where row_index < 0, in one pass."""
    x = x.contiguous()
    P, C = row_index.numel(), x.shape[1]
    q = torch.empty((P, C), dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty((P, C // 32), dtype=torch.uint8, device=x.device)
    _lib.check(_lib.load().mxgg_quantize_mx_gather(_ptr(x), _IN_DTYPES[x.dtype], x.shape[0], _ptr(row_index), P, C,
                                                   _ptr(q), _ptr(s), _stream(x.device)), "mxgg_quantize_mx_gather")
    return s, q


def combine_top2(y: Tensor, layout: DispatchLayout, weights: Tensor, out_dtype=torch.bfloat16) -> Tensor:
    """out[t] = sum_k weights[t, k] * y[pair_pos[t, k]] (fp32 sum in choice order, one pass)."""
    if out_dtype != torch.bfloat16 or y.dtype != torch.bfloat16:
        raise TypeError("combine_top2 takes and returns bf16 rows")
    y = y.contiguous()
    T, k = layout.pair_pos.shape
    N = y.shape[1]
    out = torch.empty((T, N), dtype=torch.bfloat16, device=y.device)
    pos = layout.pair_pos.to(torch.int64).contiguous()
    w = weights.to(torch.float32).contiguous()
    _lib.check(_lib.load().mxgg_combine_topk(_ptr(y), y.shape[0], _ptr(pos), _ptr(w), T, N, k, _ptr(out),
                                             _stream(y.device)), "mxgg_combine_topk")
    return out


def _quantize_weights(w: Tensor, fp4: bool):
    L, N, K = w.shape
    w2 = w.reshape(L * N, K)
    if fp4:
        s, q = to_mx_fp4(w2, _lib.SCALE_ROW_MAJOR)
        return q.view(torch.uint8).reshape(L, N, K // 2).view(torch.float4_e2m1fn_x2), s.reshape(L, N, K // 32)
    s, q = to_mx(w2, _lib.QUANT_ROWS, _lib.SCALE_ROW_MAJOR)
    return q.reshape(L, N, K), s.reshape(L, N, K // 32)


class MoELayer:
    """Top-2 MoE FFN forward with `experts` hosted on this rank.

    w_up (L, d_ff, d_model) and w_down (L, d_model, d_ff) bf16 are the hosted
    experts' weights (quantised once here); `placement`/`ep` select expert
    parallelism (None: every expert on this GPU)."""

    def __init__(self, w_up: Tensor, w_down: Tensor, n_experts: int, weights_fp4: bool = False,
                 placement: Optional[ExpertPlacement] = None, ep: Optional[FusedExpertParallel] = None):
        self.n_experts = n_experts
        self.placement = placement
        self.ep = ep
        self.d_ff, self.d_model = w_up.shape[1], w_up.shape[2]
        self.fp4 = weights_fp4
        self.up_q, self.up_s = _quantize_weights(w_up, weights_fp4)
        self.down_q, self.down_s = _quantize_weights(w_down, weights_fp4)

    def forward(self, x: Tensor, logits: Tensor) -> Tensor:
        experts, weights = route_top2(logits)
        layout = dispatch_layout(experts, self.n_experts)
        a_s, a_q = quantize_gather(x, layout.row_index)
        if self.ep is None:
            offs = torch.tensor(layout.counts, dtype=torch.int64).cumsum(0).to(torch.int32).to(x.device)
            seg_e = torch.arange(self.n_experts, dtype=torch.int32, device=x.device)
            # the up projection's epilogue writes to_mx of its bf16 output
            h_s, h_q, _, _, _ = grouped_mm_mx(a_q, self.up_q, a_s, self.up_s, offs, seg_e, torch.bfloat16, False)
            y = grouped_mm_segments(h_q, self.down_q, h_s, self.down_s, offs, seg_e, torch.bfloat16)
        else:
            # rows stream into the hosts' receive buffers while the up projection
            # consumes them; the down projection sends its rows to their owners
            ep = self.ep
            plan = ep.plan(layout.counts, self.placement)
            ep.dispatch(plan, a_q, a_s)
            h_q = torch.empty((plan.rows_recv, self.d_ff), dtype=torch.float8_e4m3fn, device=x.device)
            h_s = torch.empty((plan.rows_recv, self.d_ff // 32), dtype=torch.uint8, device=x.device)
            ep.gemm_received(plan, self.d_model, self.up_q, self.up_s, torch.bfloat16, local_mx=(h_q, h_s))
            ep.gemm_local(plan, h_q, h_s, self.down_q, self.down_s, torch.bfloat16)
            y = ep.finish(plan, self.d_model, torch.bfloat16)
        return combine_top2(y, layout, weights)

    def flops(self, tokens: int) -> float:
        """Useful FLOPs of one forward over `tokens` tokens (padding excluded)."""
        return 2.0 * (2 * tokens) * self.d_model * self.d_ff * 2
