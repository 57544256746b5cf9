"""MXFP4 (e2m1) pieces of the oracle, on CPU.

The reference has no MXFP4 path, so these pin the definitions the GPU
quantiser and the e2m1-weight GEMM are checked against: the e2m1 grid, its
round-to-nearest-even ties, saturation, NaN -> +6, FLOOR scaling with emax 2,
and the nibble packing (element 2i in the low nibble)."""
import numpy as np

from helpers import O


def test_e2m1_grid_and_ties():
    grid = np.array([0, .5, 1, 1.5, 2, 3, 4, 6], dtype=np.float32)
    assert np.array_equal(O.e2m1_decode(O.e2m1_encode(grid)), grid)
    assert np.array_equal(O.e2m1_decode(O.e2m1_encode(-grid[1:])), -grid[1:])
    # midpoints round to the even code: .25->0, .75->1, 1.25->1, 1.75->2, 2.5->2, 3.5->4, 5->4
    mids = np.array([.25, .75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)
    want = np.array([0, 1, 1, 2, 2, 4, 4], dtype=np.float32)
    assert np.array_equal(O.e2m1_decode(O.e2m1_encode(mids)), want)
    # NaN becomes +6, signed zero keeps its sign bit
    assert O.e2m1_encode(np.array([np.nan], np.float32))[0] == 7
    assert O.e2m1_encode(np.array([-0.0], np.float32))[0] == 8


def test_to_mx_e2m1_floor_scale_and_saturation():
    x = np.zeros((1, 64), np.float32)
    x[0, :32] = np.linspace(-7.0, 7.0, 32)      # amax 7 -> exponent 2 -> scale 2^(2-2) = 1
    x[0, 32] = np.inf                            # inf block saturates to 6 * 2^(126-127+...)
    s, q = O.to_mx(x, elem="e2m1")
    assert s[0, 0] == 127
    assert s[0, 1] == 255 - 2                    # exponent field 255 (inf) - emax
    d = O.dequant(q, s, elem="e2m1")
    assert np.all(np.abs(d[0, :32]) <= 6.0)
    assert d[0, 0] == -6.0 and d[0, 31] == 6.0


def test_pack_roundtrip():
    rng = np.random.default_rng(0)
    n = rng.integers(0, 16, size=(3, 64), dtype=np.uint8)
    p = O.pack_e2m1(n)
    assert p.shape == (3, 32)
    assert np.array_equal(p[0, 0] & 0xF, n[0, 0]) and np.array_equal(p[0, 0] >> 4, n[0, 1])
    assert np.array_equal(O.unpack_e2m1(p), n)
