"""The C ABI on a machine without a GPU: the library loads, exports every
symbol include/mxgg.h declares, and rejects bad arguments before touching
the device (no kernel launches here)."""
import ctypes
import os
import re

import pytest

from helpers import ROOT

import mxgg
from mxgg import _lib

HEADER = os.path.join(ROOT, "include", "mxgg.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"\b(mxgg_[a-z_0-9]+)\s*\(", text)))


def test_library_loads_and_exports_header_symbols():
    lib = _lib.load()
    syms = declared_symbols()
    assert len(syms) >= 8
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in mxgg.h but not exported"
        assert s in _lib.SIGNATURES, f"{s} has no ctypes signature"
    assert lib.mxgg_version() >= 1


def _err(rc):
    return rc, _lib.load().mxgg_last_error().decode()


def test_grouped_mm_rejects_bad_contraction():
    lib = _lib.load()
    rc, msg = _err(lib.mxgg_grouped_mm(None, None, None, None, None, 64, 64, 48, 1, ctypes.c_void_p(16), 0, None, 0, None))
    assert rc == 1 and "multiple of 32" in msg


def test_grouped_mm_rejects_bad_dtype_and_groups():
    lib = _lib.load()
    rc, msg = _err(lib.mxgg_grouped_mm(None, None, None, None, None, 64, 64, 64, 1, ctypes.c_void_p(16), 7, None, 0, None))
    assert rc == 1 and "out_dtype" in msg
    rc, msg = _err(lib.mxgg_grouped_mm(None, None, None, None, None, 64, 64, 64, 0, ctypes.c_void_p(16), 0, None, 0, None))
    assert rc == 1
    rc, msg = _err(lib.mxgg_grouped_mm(None, None, None, None, None, 64, 64, 64, 300, ctypes.c_void_p(16), 0, None, 0, None))
    assert rc == 3 and "groups" in msg


def test_grouped_mm_rejects_null_and_misaligned():
    lib = _lib.load()
    rc, msg = _err(lib.mxgg_grouped_mm(None, None, None, None, None, 64, 64, 64, 1, ctypes.c_void_p(16), 0, None, 0, None))
    assert rc == 1 and "null" in msg
    p = ctypes.c_void_p(0x1001)
    rc, msg = _err(lib.mxgg_grouped_mm(p, p, p, p, p, 64, 64, 64, 1, ctypes.c_void_p(16), 0, None, 0, None))
    assert rc == 1 and "aligned" in msg


def test_wgrad_rejects_bad_tokens():
    lib = _lib.load()
    rc, msg = _err(lib.mxgg_wgrad(None, None, None, None, None, 64, 64, 40, 2, ctypes.c_void_p(16), 0, None, 0, None))
    assert rc == 1 and "multiple of 32" in msg


def test_quantize_rejects_bad_shapes():
    lib = _lib.load()
    p = ctypes.c_void_p(0x1000)
    rc, msg = _err(lib.mxgg_quantize_mx(p, 0, 4, 48, p, p, 0, 0, None))
    assert rc == 1 and "multiple of 32" in msg
    rc, msg = _err(lib.mxgg_quantize_mx(p, 0, 40, 64, p, p, 1, 0, None))
    assert rc == 1 and "multiple of 32" in msg
    rc, msg = _err(lib.mxgg_quantize_mx(p, 9, 32, 64, p, p, 0, 0, None))
    assert rc == 1 and "x_dtype" in msg
    rc, msg = _err(lib.mxgg_quantize_mx(p, 0, 32, 64, p, p, 0, 5, None))
    assert rc == 1 and "layout" in msg


def test_workspace_size_query():
    lib = _lib.load()
    # A atoms for every 128-row slab x 128-element stage plus the B atoms, 1 KiB aligned
    n = lib.mxgg_grouped_mm_workspace_size(16640, 8192, 8192, 8)
    assert n > 0 and n % 1024 == 0
    assert n >= (16640 // 128 + 7) * 64 * 512 + 8 * 8192 // 128 * 64 * 512
    assert lib.mxgg_grouped_mm_workspace_size(-1, 8, 8, 1) == -1
    assert lib.mxgg_wgrad_workspace_size(256, 256, 1024, 4) > 0


def test_tile_config_validation():
    lib = _lib.load()
    assert lib.mxgg_set_tile_config(0, 192, 0) == 1
    assert lib.mxgg_set_tile_config(64, 128, 0) == 1
    assert lib.mxgg_set_tile_config(256, 128, 8) == 0
    assert lib.mxgg_set_tile_config(0, 0, 0) == 0


def test_schedule_validation():
    lib = _lib.load()
    assert lib.mxgg_set_schedule(3, 0) == 1
    assert lib.mxgg_set_schedule(-1, 0) == 1
    assert lib.mxgg_set_schedule(0, 1) == 1
    assert lib.mxgg_set_schedule(0, 65) == 1
    for s in (_lib.SCHED_TILES, _lib.SCHED_SPLIT_TAIL, _lib.SCHED_DEFAULT):
        assert lib.mxgg_set_schedule(s, 0) == 0
    assert lib.mxgg_set_schedule(_lib.SCHED_DEFAULT, 4) == 0
    assert lib.mxgg_set_schedule(_lib.SCHED_DEFAULT, 0) == 0


def test_wait_limit_validation():
    # the bounded-wait limit is a host setting: 1 ms .. 60 s, 0 restores 1 s
    assert _lib.wait_limit() == 1_000_000_000
    for bad in (-1, 999_999, 61_000_000_000):
        with pytest.raises(_lib.MxggError):
            _lib.set_wait_limit(bad)
    _lib.set_wait_limit(5_000_000)
    assert _lib.wait_limit() == 5_000_000
    _lib.set_wait_limit(0)
    assert _lib.wait_limit() == 1_000_000_000


def test_workspace_holds_split_tail_partials():
    # one fp32 128 x 256 partial tile for each of up to 160 CTAs, on top of
    # the packed scales, whatever the problem
    lib = _lib.load()
    for fn in (lib.mxgg_grouped_mm_workspace_size, lib.mxgg_wgrad_workspace_size):
        assert fn(256, 256, 1024, 1) >= 160 * 128 * 256 * 4
    f = lib.mxgg_grouped_mm_workspace_size
    assert f(4096, 4096, 4096, 8) > f(4096, 4096, 4096, 1)     # B scales of every group


def test_no_cpu_fallback():
    import torch
    import utils
    with pytest.raises(RuntimeError, match="CUDA"):
        utils.to_mx(torch.randn(4, 64, dtype=torch.bfloat16))
    import kernels
    if not kernels._mxfp8_available:
        with pytest.raises(NotImplementedError):
            kernels.triton_mxfp8_grouped_mm(None, torch.empty(1, 1, 1), None, None, None)


def test_grouped_mm_mx_rejects_unsupported_outputs():
    """The fused quantised outputs need N % 32 == 0, a 2-byte output type,
    aligned data buffers and, for the transposed one, M % 32 == 0; all
    checked before any device work."""
    lib = _lib.load()
    p = ctypes.c_void_p(4096)

    def call(M, N, dtype, q, s, qt, st):
        return _err(lib.mxgg_grouped_mm_mx(p, p, p, p, p, None, M, N, 64, 1, 1, 0, None, dtype, q, s, qt, st, p,
                                           1 << 20, None))

    # N = 48: blocks of 32 output columns would straddle rows
    rc, msg = call(64, 48, 0, p, p, None, None)
    assert rc == 3 and "N % 32" in msg
    # fp32 output (dtype code 2)
    rc, msg = call(64, 64, 2, p, p, None, None)
    assert rc == 3 and "bf16 or f16" in msg
    # misaligned quantised data
    rc, msg = call(64, 64, 0, ctypes.c_void_p(4097), p, None, None)
    assert rc == 1 and "16-byte aligned" in msg
    # neither an output nor a quantised buffer
    rc, msg = call(64, 64, 0, None, None, None, None)
    assert rc == 1 and "no quantised output" in msg
    # transposed output with M = 48
    rc, msg = call(48, 64, 0, None, None, p, p)
    assert rc == 1 and "M % 32" in msg


def test_library_matches_its_sources():
    """libmxgg.so carries the digest of the sources it was built from; the
    loader refuses one built from other sources (a stale build would be
    called with argument lists it does not take)."""
    lib = _lib.load()
    assert lib.mxgg_build_id().decode() == _lib.source_digest()


def test_loader_refuses_a_stale_library(monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "source_digest", lambda: "0" * 16)
    with pytest.raises(_lib.MxggError, match="built from other sources"):
        _lib.load()


def test_eager_fast_path_conditions():
    """Plain eager calls skip the torch.library dispatcher; tracing modes,
    tensor subclasses and autograd inputs take the registered op."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode
    from mxgg import ops
    x = torch.zeros(4)
    assert ops._eager((x, 3, torch.bfloat16))
    assert not ops._eager((torch.zeros(4, requires_grad=True),))
    assert not ops._eager((torch.nn.Parameter(torch.zeros(4)),))
    with FakeTensorMode():
        assert not ops._eager((x,))


def test_fake_mode_uses_the_registered_fake_kernel():
    """Under FakeTensorMode (what torch.compile traces with) the entry points
    return shape-correct fakes without touching the library or a GPU."""
    import torch
    from torch._subclasses.fake_tensor import FakeTensorMode
    from mxgg import ops
    with FakeTensorMode():
        a = torch.empty(1024, 512, dtype=torch.float8_e4m3fn, device="cuda")
        b = torch.empty(4, 256, 512, dtype=torch.float8_e4m3fn, device="cuda")
        sa = torch.empty(1024, 16, dtype=torch.uint8, device="cuda")
        sb = torch.empty(4, 256, 16, dtype=torch.uint8, device="cuda")
        offs = torch.empty(4, dtype=torch.int32, device="cuda")
        out = ops.grouped_mm(a, b, sa, sb, offs, torch.bfloat16)
        s, q, st, qt, o = ops.grouped_mm_mx(a, b, sa, sb, offs, None, torch.bfloat16, False, True, True)
        go = torch.empty(256, 1024, dtype=torch.float8_e4m3fn, device="cuda")
        gs = torch.empty(256, 32, dtype=torch.uint8, device="cuda")
        w = ops.wgrad(go, gs, go, gs, offs, torch.float32)
    assert out.shape == (1024, 256) and out.dtype == torch.bfloat16
    assert s.shape == (1024, 8) and q.shape == (1024, 256) and st.shape == (256, 32) and qt.shape == (256, 1024)
    assert o.numel() == 0
    assert w.shape == (4, 256, 256) and w.dtype == torch.float32
