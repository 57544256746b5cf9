"""The fused expert-parallel path's routing arithmetic (`fused_layout`),
simulated on CPU for every rank of a world: the copies, the in-place self
rows and the receive-segment tables must move every row to the rank hosting
its expert and send every output row back to its owner's exact position; the
senders' atom offsets must match each receiver's own tile numbering."""
import random

import pytest

from mxgg.ep import ExpertPlacement, fused_layout


def _cases():
    rng = random.Random(7)
    out = []
    for world in (2, 3, 4, 8):
        for E in (1, 2, 4, 8, 16, 24):
            if (E >= world and E % world) or (E < world and world % E):
                continue
            for align in (32, 16):
                C = [[rng.randint(0, 12) * align for _ in range(E)] for _ in range(world)]
                if world > 1:
                    C[1][0] = 0
                out.append((world, E, align, C))
    return out


@pytest.mark.parametrize("piece_rows", [2048, 64])
@pytest.mark.parametrize("world,E,align,C", _cases())
def test_fused_layout_moves_every_row(world, E, align, C, piece_rows):
    """piece_rows 64 cuts most peer blocks into pieces (up to four each)."""
    pl = ExpertPlacement(world, E)
    lays = [fused_layout(C, pl, r, piece_rows=piece_rows) for r in range(world)]
    # each rank's local rows, tagged (owner, local row, expert)
    local = []
    for s in range(world):
        rows = []
        for e in range(E):
            rows += [(s, len(rows) + i, e) for i in range(C[s][e])]
        local.append(rows)
    # receive buffers: peers' copies; a rank's own slot stays empty (read in place)
    recv = [[None] * lays[d]["rows_recv"] for d in range(world)]
    slot_of = [[None] * lays[d]["rows_recv"] for d in range(world)]   # flag slot raised after the row's copy
    for s in range(world):
        for (d, dst_row, src_row, rows, slot) in lays[s]["copies"]:
            assert d != s and rows > 0
            assert slot % world == s and 0 <= slot < 32
            recv[d][dst_row:dst_row + rows] = local[s][src_row:src_row + rows]
            slot_of[d][dst_row:dst_row + rows] = [slot] * rows
    for d in range(world):
        lay = lays[d]
        seg = lay["seg"]
        assert lay["rows_recv"] == lay["need_recv"][d]
        lo = 0
        g_cum = 0          # 128-row scale slabs of the segments so far
        first_slab = {}
        for i, hi in enumerate(seg["offs"]):
            sid, le = seg["src"][i], seg["expert"][i]
            src = sid % world
            assert seg["dst"][i] == src
            e = pl.experts_of(d)[le]
            first_slab.setdefault(src, g_cum)
            for k, r in enumerate(range(lo, hi)):
                row = local[d][lay["self_base"] + r] if src == d else recv[d][r]
                assert row is not None, "a received row was never copied"
                if src != d:
                    # the segment waits on the flag raised after this very row's copy
                    assert slot_of[d][r] == sid
                owner, lrow, ex = row
                assert owner == src and ex == e
                # the output row goes back to its owner's exact position
                assert seg["dst_row"][i] + k == lrow
                assert seg["local_row"][i] == lo
            g_cum += (hi - lo + 127) // 128
            lo = hi
        # pieces cut segments only on their 256-row tile grid: the 128-row scale
        # slabs (and the GEMM's tiles) are those of the uncut segments
        uncut = 0
        for s in range(world):
            for e in pl.experts_of(d):
                if pl.dest(s, e) == d:
                    uncut += (C[s][e] + 127) // 128
        assert g_cum == uncut
        # every row routed to d arrived exactly once
        want = sorted(r for s in range(world) for r in local[s] if pl.dest(s, r[2]) == d)
        got = sorted(local[d][lay["self_base"] + r] if seg["src"][i] == d else recv[d][r]
                     for i, hi in enumerate(seg["offs"])
                     for r in range(seg["offs"][i - 1] if i else 0, hi))
        assert got == want
        # senders pack their scale atoms where d's slab numbering puts their first segment
        for s in range(world):
            for (dd, cum, m0, src_row, rows) in lays[s]["pack"]:
                if dd == d:
                    assert m0 == first_slab[s]
                    assert cum[-1] == rows
    # inbox blocks: exactly the 32-row blocks of rows computed by other ranks
    for r in range(world):
        lay = lays[r]
        if not lay["inbox_ok"]:
            assert not all(c % 32 == 0 for row in C for c in row)
            continue
        remote = {i // 32 for i, (_, _, e) in enumerate(local[r]) if pl.dest(r, e) != r}
        assert set(lay["remote_blocks"]) == remote


def test_pieces_cut_large_blocks_on_the_tile_grid():
    from mxgg.ep import _piece_cuts
    # one segment of 16640 rows: four pieces, cuts on multiples of 256
    cuts = _piece_cuts([16640], 4)
    assert cuts == [4352, 8448, 12544]
    # a cut moves forward to the next multiple of 256 rows past its segment's start ...
    assert _piece_cuts([100, 5000], 2) == [2660]
    # ... or, when the segment ends first, to the next segment's start
    assert _piece_cuts([1000, 100, 1000], 2) == [1100]
    # blocks too short for pieces stay whole
    assert _piece_cuts([300], 1) == []
    pl = ExpertPlacement(2, 2)
    C = [[1280, 15360], [15360, 1280]]
    lay = fused_layout(C, pl, 0)
    # rank 0 sends 15360 rows to rank 1 in four flagged pieces, slots 0, 2, 4, 6
    assert [c[4] for c in lay["copies"]] == [0, 2, 4, 6]
    assert sum(c[3] for c in lay["copies"]) == 15360
    # it receives rank 1's 15360 rows in four pieces; its own 1280 rows stay whole
    assert lay["seg"]["src"] == [0, 1, 3, 5, 7]


@pytest.mark.parametrize("N,K,want", [(5120, 5120, 2560), (8192, 5120, 3584), (8192, 8192, 4096),
                                      (5120, 8192, 2304), (2048, 2048, None), (2048, 8192, None)])
def test_wgrad_split_rows(N, K, want):
    """The cut of the overlapped replica sum: on the 256-row tile grid, no
    extra round of tiles over 74 CTA pairs, nearest the middle; small grids
    are not cut."""
    from mxgg.ep import wgrad_split_rows
    P = 74
    cut = wgrad_split_rows(1, N, K, P)
    assert cut == want
    if cut is not None:
        nt, kt = N // 256, K // 256
        a = cut // 256
        assert cut % 256 == 0 and 0 < cut < N
        assert -(-a * kt // P) + -(-(nt - a) * kt // P) <= -(-nt * kt // P)
    assert wgrad_split_rows(2, N, K, P) is None          # several local experts: one launch
