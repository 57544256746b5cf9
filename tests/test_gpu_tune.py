"""The autotune harness on the GPU: it times candidate configs on a small
point, returns a table entry for each call shape, and an installed table
changes the config a call runs with but not its results (rel-L2 <= 1e-3
against the oracle, as every forward)."""
import numpy as np
import pytest
import torch

from helpers import O, bf16_round, f32, gpu_status_clear, u8

pytestmark = pytest.mark.gpu


def test_tune_small_points_and_install():
    import kernels
    import utils
    from mxgg import _lib, tune
    gpu_status_clear()
    shapes = [(2, 1024, 256, 512)]
    cfgs = [tune.Config(256, 256, 16, _lib.SCHED_SPLIT_TAIL), tune.Config(128, 128, 2, _lib.SCHED_TILES)]
    table = tune.tune(shapes, ["fwd", "wgrad"], cfgs, gpus=1, reps=3)
    fwd = table.lookup("fwd", 2, 256, 512)
    assert fwd in cfgs and table.lookup("wgrad", 2, 256, 512) in cfgs
    assert table.device and all(us > 0 for (_, us, _) in table.entries.values())
    # force the single-CTA config through a table and check the numbers
    forced = tune.Table()
    forced.add("fwd", 2, 256, 512, cfgs[1], 1.0)
    g = torch.Generator().manual_seed(3)
    a_s, a_q = utils.to_mx(torch.randn(1024, 512, generator=g).to(torch.bfloat16).cuda())
    b_s, b_q = utils.to_mx((torch.randn(2, 256, 512, generator=g) * 0.05).to(torch.bfloat16).cuda())
    offs = torch.tensor([300, 1024], dtype=torch.int32, device="cuda")
    try:
        tune.install(forced)
        out = kernels.triton_mxfp8_grouped_mm(a_q, b_q, a_s, b_s, offs)
    finally:
        tune.install(None)
    torch.cuda.synchronize()
    ref = O.grouped_mm(u8(a_q), u8(a_s), u8(b_q), u8(b_s), offs.cpu().numpy(), acc=np.float32)
    assert O.rel_l2(f32(out), bf16_round(ref)) <= 1e-3
    assert gpu_status_clear() == 0
