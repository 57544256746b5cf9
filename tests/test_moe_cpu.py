"""Routing layout of the MoE layer on CPU: top-2 choices sorted by expert,
every expert's rows padded to a multiple of 32, positions consistent."""
import torch

from mxgg.moe import dispatch_layout, route_top2


def test_route_top2_weights_sum_to_one():
    g = torch.Generator().manual_seed(0)
    logits = torch.randn(64, 8, generator=g)
    e, w = route_top2(logits)
    assert e.shape == (64, 2) and torch.all(e[:, 0] != e[:, 1])
    assert torch.allclose(w.sum(-1), torch.ones(64))
    assert torch.all(w[:, 0] >= w[:, 1])


def test_dispatch_layout():
    g = torch.Generator().manual_seed(1)
    T, E = 200, 6
    e, _ = route_top2(torch.randn(T, E, generator=g))
    lay = dispatch_layout(e, E)
    counts = torch.bincount(e.reshape(-1), minlength=E)
    assert all(c % 32 == 0 for c in lay.counts)
    assert [int(c) for c in lay.counts] == [int((x + 31) // 32 * 32) for x in counts]
    assert lay.row_index.numel() == sum(lay.counts)
    # every (token, choice) sits in its expert's padded block and points back at its token
    starts = torch.tensor([0] + lay.counts).cumsum(0)
    for t in range(T):
        for k in range(2):
            p = int(lay.pair_pos[t, k])
            ex = int(e[t, k])
            assert starts[ex] <= p < starts[ex + 1]
            assert int(lay.row_index[p]) == t
    # the padding rows are exactly the unused ones
    assert int((lay.row_index < 0).sum()) == sum(lay.counts) - 2 * T
