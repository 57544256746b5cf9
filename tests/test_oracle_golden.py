"""The CPU oracle against vectors produced by the reference's own code.

These run without a GPU: they pin the oracle before any kernel is compared
with it.
"""
import numpy as np
import pytest

from oracle import mx_oracle as O


def _f32_from_bf16(bits):
    return O.bf16_bits_to_f32(bits)


@pytest.mark.parametrize("name,kind", [("tomx_bf16", "bf16"), ("tomx_edge", "f32"), ("tomx_f32", "f32")])
def test_to_mx_bit_exact(golden, name, kind):
    xb = golden[name + "_x"]
    x = _f32_from_bf16(xb) if kind == "bf16" else xb.view(np.float32)
    s, q = O.to_mx(x)
    np.testing.assert_array_equal(s, golden[name + "_s"])
    np.testing.assert_array_equal(q, golden[name + "_q"])


def test_to_mx_config1_inputs(golden):
    a = _f32_from_bf16(golden["fwd1_a_bits"])
    s, q = O.to_mx(a)
    np.testing.assert_array_equal(s, golden["fwd1_a_s"])
    np.testing.assert_array_equal(q, golden["fwd1_a_q"])
    b = _f32_from_bf16(golden["fwd1_b_bits"])
    s, q = O.to_mx(b)
    np.testing.assert_array_equal(s, golden["fwd1_b_s"])
    np.testing.assert_array_equal(q, golden["fwd1_b_q"])


def test_jagged_offsets_sequence(golden):
    got = np.concatenate(O.llama4_offsets(123))
    np.testing.assert_array_equal(got, golden["llama4_offs"])
    lens = [len(o) for o in O.llama4_offsets(123)]
    np.testing.assert_array_equal(lens, golden["llama4_offs_lens"])


def test_product_jagged_offsets_sequence(golden):
    """The product's generate_jagged_offs (the one bench.py draws with) replays
    the reference bench's seeded sequence: random.seed(123), then one draw per
    Llama4 shape in the reference's order (bench.py:243-257)."""
    import random

    import utils
    random.seed(123)
    draws = [utils.generate_jagged_offs(e, m, 32, device="cpu").numpy() for (e, m, n, k) in O.llama4_shapes()]
    np.testing.assert_array_equal(np.concatenate(draws), golden["llama4_offs"])
    np.testing.assert_array_equal([len(d) for d in draws], golden["llama4_offs_lens"])


def test_grouped_mm_emulation(golden):
    out = O.grouped_mm(golden["fwd1_a_q"], golden["fwd1_a_s"], golden["fwd1_b_q"],
                       golden["fwd1_b_s"], golden["fwd1_offs"])
    ref = golden["fwd1_out_f32"]
    valid = ~np.isnan(ref)
    assert O.rel_l2(out[valid], ref[valid]) < 1e-6
    # the quantised result keeps the reference's SQNR gate against bf16 hp
    hp = O.bf16_bits_to_f32(golden["fwd1_hp_bf16"])
    assert O.compute_error(hp, out) >= 27.0


def test_wgrad_emulation(golden):
    out = O.wgrad(golden["wg_go_q"], golden["wg_go_s"], golden["wg_ia_q"],
                  golden["wg_ia_s"], golden["wg_offs"])
    assert O.rel_l2(out, golden["wg_out_f32"]) < 1e-6


def test_e4m3_roundtrip_all_codes():
    codes = np.arange(256, dtype=np.uint8)
    vals = O.e4m3_decode(codes)
    ok = ~np.isnan(vals)
    back = O.e4m3_encode(vals[ok])
    np.testing.assert_array_equal(back, codes[ok])


def test_e2m1_roundtrip_all_codes():
    codes = np.arange(16, dtype=np.uint8)
    back = O.e2m1_encode(O.e2m1_decode(codes))
    # -0 encodes as 8, +0 as 0
    np.testing.assert_array_equal(back, codes)


def test_tile_map_restatement():
    hist, raw, pad, pmap = O.build_tile_map([100, 100, 356, 1000], 1000, 128)
    assert list(hist) == [100, 0, 256, 644]
    assert list(raw) == [0, 100, 100, 356]
    assert int(pad) == 1 + 0 + 2 + 6
    assert len(pmap) == 8 + 3
    assert list(pmap[:9]) == [0, (0 << 16) | 2, (1 << 16) | 2] + [(i << 16) | 3 for i in range(6)]
    assert list(pmap[9:]) == [-1, -1]
