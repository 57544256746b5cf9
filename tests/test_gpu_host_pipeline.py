"""mxgg.host.HostPipeline: grouped GEMMs on pinned host operands, cut into
pieces on three streams, give the same bits as one call of the entry point
on device copies of the operands (whole-tile schedule): forward split by
groups (several experts) and by rows (one expert), dgrad's layout, empty
groups, and wgrad split by rows of go_t."""
import pytest
import torch

from helpers import gpu_status_clear, offsets, randn_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _status():
    gpu_status_clear()
    yield
    assert gpu_status_clear() == 0, "a device-side wait timed out"


def _pin(t):
    return t.cpu().contiguous().pin_memory()


@pytest.mark.parametrize("pieces", [1, 3, 4])
@pytest.mark.parametrize("E,M,N,K,empty", [(4, 4096, 768, 512, False), (1, 2976, 512, 384, False),
                                           (6, 2048, 256, 1024, True)])
def test_forward_from_host_matches_device_call(pieces, E, M, N, K, empty):
    import kernels
    import utils
    from mxgg.host import HostPipeline
    if empty:
        ends = [0, 512, 512, 1024, 2000, M]          # empty groups, one at the front
    else:
        ends = offsets(E, M, 32, seed=E + M)
    offs = torch.tensor(ends, dtype=torch.int32, device="cuda")
    a_s, a_q = utils.to_mx(randn_bf16((M, K), seed=1))
    w_s, w_q = utils.to_mx(randn_bf16((E, N, K), seed=2, scale=0.05))
    want = kernels.triton_mxfp8_grouped_mm(a_q, w_q, a_s, w_s, offs)
    out = torch.empty((M, N), dtype=torch.bfloat16).pin_memory()
    hp = HostPipeline(pieces=pieces)
    hp.grouped_mm(_pin(a_q), _pin(w_q), _pin(a_s), _pin(w_s), ends, out)
    torch.cuda.synchronize()
    assert torch.equal(out, want.cpu())
    # a second call through the same pipeline (staging buffers reused) on other operands
    a2_s, a2_q = utils.to_mx(randn_bf16((M, K), seed=3))
    want2 = kernels.triton_mxfp8_grouped_mm(a2_q, w_q, a2_s, w_s, offs)
    hp.grouped_mm(_pin(a2_q), _pin(w_q), _pin(a2_s), _pin(w_s), torch.tensor(ends), out)
    torch.cuda.synchronize()
    assert torch.equal(out, want2.cpu())


@pytest.mark.parametrize("pieces", [1, 4])
@pytest.mark.parametrize("E,M,N,K", [(3, 2048, 1280, 768), (1, 1024, 512, 256)])
def test_wgrad_from_host_matches_device_call(pieces, E, M, N, K):
    import kernels
    import utils
    from mxgg.host import HostPipeline
    ends = offsets(E, M, 32, seed=7)
    offs = torch.tensor(ends, dtype=torch.int32, device="cuda")
    go_s, go_q = utils.to_mx_dim1(randn_bf16((M, N), seed=4))
    x_s, x_q = utils.to_mx_dim1(randn_bf16((M, K), seed=5))
    want = kernels.triton_mxfp8_wgrad(go_q, go_s, x_q, x_s, offs)
    out = torch.empty((E, N, K), dtype=torch.bfloat16).pin_memory()
    HostPipeline(pieces=pieces).wgrad(_pin(go_q), _pin(go_s), _pin(x_q), _pin(x_s), ends, out)
    torch.cuda.synchronize()
    assert torch.equal(out, want.cpu())


def test_host_pipeline_rejects_device_or_pageable_operands():
    from mxgg.host import HostPipeline
    hp = HostPipeline()
    a = torch.zeros(64, 64, dtype=torch.uint8)
    with pytest.raises(ValueError):
        hp.grouped_mm(a, a.view(1, 64, 64), a, a.view(1, 64, 64), [64],
                      torch.empty(64, 64, dtype=torch.bfloat16).pin_memory())
