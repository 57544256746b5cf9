"""Piece planning of mxgg.host.HostPipeline (no GPU): the pieces of a
forward call cover every group and row once, in order, with their relative
group ends summing to the piece's rows; wgrad row cuts sit on the 256-row
tile grid."""
import random

import pytest

from mxgg.host import group_pieces, row_cuts


def _check(ends, pieces):
    E, M = len(ends), ends[-1]
    ps = group_pieces(ends, 512 + 16, 1 << 20, pieces)
    assert 1 <= len(ps) <= max(1, pieces)
    assert ps[0][0] == 0 and ps[0][2] == 0 and ps[-1][1] == E and ps[-1][3] == M
    by_groups = E >= 2 and pieces > 1
    for (g0, g1, r0, r1), nxt in zip(ps, ps[1:] + [None]):
        assert g0 < g1 and r0 <= r1
        if nxt is not None:
            assert nxt[2] == r1
            assert nxt[0] == (g1 if by_groups else 0)
        if by_groups:
            # runs of whole groups: the rows are exactly those groups' rows
            assert r0 == (ends[g0 - 1] if g0 else 0) and r1 == ends[g1 - 1]
        else:
            # runs of rows over every group
            assert (g0, g1) == (0, E)
        rel = [min(max(ends[g] - r0, 0), r1 - r0) for g in range(g0, g1)]
        assert rel == sorted(rel) and rel[-1] == r1 - r0


@pytest.mark.parametrize("pieces", [1, 2, 4, 8])
def test_group_pieces_cover_every_row_once(pieces):
    rng = random.Random(pieces)
    for E in (1, 2, 3, 8, 16):
        for _ in range(20):
            M = 32 * rng.randint(E, 600)
            ends = sorted(rng.sample(range(0, M + 1, 32), E - 1)) + [M] if E > 1 else [M]
            _check(ends, pieces)
    _check([0, 0, 4096, 4096], 4)          # empty groups, first and last


def test_row_cuts_on_the_tile_grid():
    assert row_cuts(8192, 4) == [0, 2048, 4096, 6144, 8192]
    assert row_cuts(5120, 8) == [0, 512, 1280, 1792, 2560, 3072, 3840, 4352, 5120]
    assert row_cuts(300, 4) == [0, 300]
    for rows in (256, 1000, 2976, 16640):
        for p in (1, 3, 8):
            c = row_cuts(rows, p)
            assert c[0] == 0 and c[-1] == rows and c == sorted(set(c))
            assert all(x % 256 == 0 for x in c[1:-1])
