"""The torch restatement of the reference's CPU path (oracle/cpu_path.py),
which bench.py times as the CPU baseline and the reference arm, pinned to
vectors the reference's own code produced (tests/golden/make_golden.py)."""
import numpy as np
import pytest
import torch

from oracle import cpu_path as C
from oracle import mx_oracle as O


def _bf16(bits):
    return torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("name,kind", [("tomx_bf16", "bf16"), ("tomx_edge", "f32"), ("tomx_f32", "f32")])
def test_to_mx_cpu_matches_reference_vectors(golden, name, kind):
    xb = golden[name + "_x"]
    x = _bf16(xb) if kind == "bf16" else torch.from_numpy(xb.view(np.float32).copy())
    s, q = C.to_mx_cpu(x)
    np.testing.assert_array_equal(s.numpy(), golden[name + "_s"])
    np.testing.assert_array_equal(q.view(torch.uint8).numpy(), golden[name + "_q"])


def test_forward_and_wgrad_match_reference_outputs(golden):
    a = _bf16(golden["fwd1_a_bits"])
    b = _bf16(golden["fwd1_b_bits"])
    a_s, a_q = C.to_mx_cpu(a)
    b_s, b_q = C.to_mx_cpu(b)
    np.testing.assert_array_equal(a_s.numpy(), golden["fwd1_a_s"])
    out = C.grouped_mm_cpu(C.dequant_cpu(a_q, a_s), C.dequant_cpu(b_q, b_s), golden["fwd1_offs"].tolist())
    ref = golden["fwd1_out_f32"]
    ok = ~np.isnan(ref)
    assert O.rel_l2(out.numpy()[ok], ref[ok]) < 1e-6
    go = C.dequant_cpu(torch.from_numpy(golden["wg_go_q"]).view(torch.float8_e4m3fn), torch.from_numpy(golden["wg_go_s"]))
    ia = C.dequant_cpu(torch.from_numpy(golden["wg_ia_q"]).view(torch.float8_e4m3fn), torch.from_numpy(golden["wg_ia_s"]))
    dw = C.wgrad_cpu(go, ia, golden["wg_offs"].tolist())
    assert O.rel_l2(dw.numpy(), golden["wg_out_f32"]) < 1e-6


def test_offsets_draw_matches_reference_sequence(golden):
    import random
    rng = random.Random(123)
    draws = [C.draw_offs(e, m, 32, rng) for (e, m, n, k) in O.llama4_shapes()]
    np.testing.assert_array_equal(np.concatenate(draws), golden["llama4_offs"])


def test_sample_runs_every_pass():
    s = C.CpuPathSample(threads=2, shapes=[(2, 64, 64)], M=256)
    assert [p[0] for p in s.points] == ["fwd", "dgrad", "wgrad"]
    assert all(s.run_point(i) > 0 for i in range(3))
    assert "to_mx" in s.describe()
