"""Autotune harness host logic (no GPU): the candidate space, per-call
configs through the C ABI, best-config selection, dealing points to GPUs,
and the table's JSON round trip, merge and lookup."""
import json
import os
import tempfile

import pytest

from helpers import ROOT  # noqa: F401  (puts the package on sys.path)
from mxgg import _lib, tune


def test_config_space_is_valid_and_distinct():
    space = tune.config_space()
    assert len(space) == len(set(space)) == 24
    assert all(c.valid() for c in space)
    assert {(c.tile_m, c.tile_n) for c in space} == {(256, 256), (256, 128), (128, 256), (128, 128)}
    assert not tune.Config(tile_m=192).valid() and not tune.Config(split_max=1).valid()


def test_call_config_is_passed_per_call(monkeypatch):
    # a tuned config travels with the call: nothing process-wide is touched
    def boom(*a):
        raise AssertionError("process-wide setter called")
    monkeypatch.setattr(_lib, "set_tile_config", boom)
    monkeypatch.setattr(_lib, "set_schedule", boom)
    assert tune.call_config(None) is None
    assert tune.call_config(tune.Config(128, 256, 4, _lib.SCHED_TILES, 0)) == [128, 256, 4, _lib.SCHED_TILES, 0]
    with pytest.raises(ValueError):
        tune.call_config(tune.Config(tile_n=64))


def test_wrappers_pass_the_installed_entry(monkeypatch):
    import torch

    import kernels
    import mxgg
    from kernels import backward, forward
    seen = {}
    monkeypatch.setattr(forward, "_mxfp8_available", True)
    monkeypatch.setattr(backward, "_mxfp8_available", True)
    # the wrappers pass (..., cfg, scale_layout)
    monkeypatch.setattr(mxgg.ops, "grouped_mm", lambda *a: seen.setdefault("fwd", a[-2:]))
    monkeypatch.setattr(mxgg.ops, "wgrad", lambda *a: seen.setdefault("wgrad", a[-2:]))
    t = tune.Table()
    t.add("fwd", 2, 256, 512, tune.Config(128, 128, 2, _lib.SCHED_TILES, 0), 1.0)
    t.add("wgrad", 2, 256, 512, tune.Config(256, 256, 8, _lib.SCHED_SPLIT_TAIL, 3), 1.0)
    tune.install(t)
    try:
        a = torch.zeros(64, 512, dtype=torch.float8_e4m3fn)
        b = torch.zeros(2, 256, 512, dtype=torch.float8_e4m3fn)
        offs = torch.tensor([32, 64], dtype=torch.int32)
        kernels.triton_mxfp8_grouped_mm(a, b, torch.zeros(64, 16, dtype=torch.uint8),
                                        torch.zeros(2, 256, 16, dtype=torch.uint8), offs)
        kernels.triton_mxfp8_wgrad(torch.zeros(256, 64, dtype=torch.float8_e4m3fn), torch.zeros(256, 2, dtype=torch.uint8),
                                   torch.zeros(512, 64, dtype=torch.float8_e4m3fn), torch.zeros(512, 2, dtype=torch.uint8),
                                   offs)
    finally:
        tune.install(None)
    assert seen == {"fwd": ([128, 128, 2, _lib.SCHED_TILES, 0], _lib.SCALE_ROW_MAJOR),
                    "wgrad": ([256, 256, 8, _lib.SCHED_SPLIT_TAIL, 3], _lib.SCALE_ROW_MAJOR)}


def test_wrappers_pass_the_scale_layout(monkeypatch):
    import torch

    import kernels
    import mxgg
    from kernels import backward, forward
    seen = {}
    monkeypatch.setattr(forward, "_mxfp8_available", True)
    monkeypatch.setattr(backward, "_mxfp8_available", True)
    monkeypatch.setattr(mxgg.ops, "grouped_mm", lambda *a: seen.setdefault("fwd", a[-1]))
    monkeypatch.setattr(mxgg.ops, "wgrad", lambda *a: seen.setdefault("wgrad", a[-1]))
    a = torch.zeros(64, 512, dtype=torch.float8_e4m3fn)
    b = torch.zeros(2, 256, 512, dtype=torch.float8_e4m3fn)
    offs = torch.tensor([32, 64], dtype=torch.int32)
    kernels.triton_mxfp8_grouped_mm(a, b, torch.zeros(1, dtype=torch.uint8), torch.zeros(1, dtype=torch.uint8), offs,
                                    scale_layout="blocked")
    kernels.triton_mxfp8_wgrad(torch.zeros(256, 64, dtype=torch.float8_e4m3fn), torch.zeros(1, dtype=torch.uint8),
                               torch.zeros(512, 64, dtype=torch.float8_e4m3fn), torch.zeros(1, dtype=torch.uint8),
                               offs, scale_layout="blocked")
    assert seen == {"fwd": _lib.SCALE_BLOCKED, "wgrad": _lib.SCALE_BLOCKED}
    with pytest.raises(ValueError, match="scale_layout"):
        kernels.triton_mxfp8_grouped_mm(a, b, torch.zeros(1, dtype=torch.uint8), torch.zeros(1, dtype=torch.uint8),
                                        offs, scale_layout="swizzled")


def test_library_rejects_a_bad_call_config():
    # validated before any device work, so no GPU is needed
    lib = _lib.load()
    for bad, word in [((64, 0, 0, 0, 0), "tile_m"), ((0, 96, 0, 0, 0), "tile_n"), ((0, 0, -1, 0, 0), "group_m"),
                      ((0, 0, 0, 7, 0), "schedule"), ((0, 0, 0, 0, 1), "split_max")]:
        rc = lib.mxgg_grouped_mm_cfg(None, None, None, None, None, 128, 128, 128, 1, None, _lib.DTYPE_BF16,
                                     _lib.gemm_config(bad), None, 0, None)
        assert rc == 1 and word in lib.mxgg_last_error().decode()
    rc = lib.mxgg_grouped_mm_cfg(None, None, None, None, None, 128, 128, 128, 1, None, _lib.DTYPE_BF16,
                                 _lib.gemm_config(None, 7), None, 0, None)
    assert rc == 1 and "scale_layout" in lib.mxgg_last_error().decode()
    cfg = _lib.GemmConfig(0, 0, 0, 0, 0)
    cfg.reserved[1] = 5
    rc = lib.mxgg_wgrad_cfg(None, None, None, None, None, 128, 128, 128, 1, None, _lib.DTYPE_BF16,
                            __import__("ctypes").pointer(cfg), None, 0, None)
    assert rc == 1 and "reserved" in lib.mxgg_last_error().decode()
    with pytest.raises(_lib.MxggError):
        _lib.set_tile_config(64, 0, 0)
    _lib.set_tile_config(0, 0, 0)


def test_tune_point_picks_the_fastest_and_skips_rejected():
    cfgs = tune.config_space()[:5]
    fake = {tuple(c.as_list()): t for c, t in [(cfgs[0], 3.0), (cfgs[1], 1.0), (cfgs[2], 1.0), (cfgs[4], 2.0)]}
    current = {}

    def run(cfg):
        current["cfg"] = tuple(cfg)

    def timer(fn):
        fn()
        c = current["cfg"]
        if c not in fake:
            raise _lib.MxggError("rejected")
        return fake[c]

    times = tune.tune_point(run, cfgs, timer)
    assert cfgs[3] not in times and len(times) == 4
    assert tune.best(times) == (cfgs[1], 1.0)      # tie with cfgs[2]: the first tried wins


def test_call_points_fold_dgrad_into_forward_calls():
    shapes = [(8, 16640, 2048, 5120), (8, 16640, 5120, 2048)]
    pts = tune.call_points(shapes, ["fwd", "dgrad", "wgrad"])
    # dgrad of (2048, 5120) is the forward call (5120, 2048), which the second point has already
    assert pts == [("fwd", 8, 16640, 2048, 5120), ("fwd", 8, 16640, 5120, 2048), ("wgrad", 8, 16640, 2048, 5120),
                   ("wgrad", 8, 16640, 5120, 2048)]
    with pytest.raises(ValueError):
        tune.call_points(shapes, ["bwd"])


def test_shard_deals_every_point_once():
    pts = tune.call_points(tune.llama4_shapes(), tune.PASSES)
    assert len(tune.llama4_shapes()) == 36
    got = sorted(p for r in range(8) for p in tune.shard(pts, r, 8))
    assert got == sorted(pts)
    assert max(len(tune.shard(pts, r, 8)) for r in range(8)) - min(len(tune.shard(pts, r, 8)) for r in range(8)) <= 1


def test_table_round_trip_merge_and_lookup():
    a = tune.Table("B200")
    a.add("fwd", 8, 2048, 5120, tune.Config(256, 256, 16, _lib.SCHED_SPLIT_TAIL), 120.0)
    a.add("fwd", 8, 2048, 5120, tune.Config(128, 256, 2, _lib.SCHED_TILES), 130.0)   # slower: ignored
    b = tune.Table("B200")
    b.add("wgrad", 1, 8192, 8192, tune.Config(256, 128, 8, _lib.SCHED_TILES), 900.0)
    b.add("fwd", 8, 2048, 5120, tune.Config(256, 128, 32, _lib.SCHED_TILES), 110.0)   # faster: wins
    a.merge(b)
    d = tempfile.mkdtemp()
    try:
        path = os.path.join(d, "t.json")
        a.save(path)
        with open(path) as f:
            assert len(json.load(f)["entries"]) == 2
        t = tune.Table.load(path)
    finally:
        for f in os.listdir(d):
            os.remove(os.path.join(d, f))
        os.rmdir(d)
    assert t.lookup("fwd", 8, 2048, 5120) == tune.Config(256, 128, 32, _lib.SCHED_TILES)
    assert t.lookup("wgrad", 1, 8192, 8192) == tune.Config(256, 128, 8, _lib.SCHED_TILES)
    assert t.lookup("fwd", 4, 2048, 5120) is None
    with pytest.raises(ValueError):
        tune.Table.from_json({"entries": [{"pass": "fwd", "E": 1, "N": 1, "K": 1, "us": 1.0,
                                           "config": {"tile_m": 96}}]})


def test_packaged_default_table(monkeypatch):
    # the packaged table: valid configs for sweep shapes only (points where
    # the library's own choice was not beaten carry no entry)
    t = tune.Table.load(tune.DEFAULT_TABLE)
    sweep = {(E, N, K) for (E, M, N, K) in tune.llama4_shapes()}
    assert t.entries
    for (ps, E, N, K), (cfg, us, M) in t.entries.items():
        assert ps in ("fwd", "wgrad") and (E, N, K) in sweep and cfg.valid() and us > 0
    (ps, E, N, K), (cfg, _, _) = sorted(t.entries.items())[0]
    # installed at import unless MXGG_TUNE_TABLE says otherwise
    monkeypatch.delenv("MXGG_TUNE_TABLE", raising=False)
    try:
        tune.install_default()
        assert tune.pick(ps, E, N, K) == cfg
        monkeypatch.setenv("MXGG_TUNE_TABLE", "none")
        tune.install_default()
        assert tune.pick(ps, E, N, K) is None
    finally:
        tune.install(None)


def test_worth_keeping_needs_a_confirmed_margin():
    a, b = tune.Config(128, 256, 2, _lib.SCHED_TILES), tune.Config(256, 256, 8, _lib.SCHED_SPLIT_TAIL)
    times = {tune.DEFAULT: 1.00, a: 0.90, b: 0.99}
    assert tune.worth_keeping(times) == (a, 0.90)
    # the second measurement must agree
    assert tune.worth_keeping(times, confirm=lambda c: (0.95, 0.96)) is None
    assert tune.worth_keeping(times, confirm=lambda c: (0.91, 1.00)) == (a, 0.90)
    # within the margin of the library's choice: no entry
    assert tune.worth_keeping({tune.DEFAULT: 1.00, a: 0.98}) is None
    assert tune.worth_keeping({tune.DEFAULT: 1.00, a: 1.10}) is None


def test_install_and_pick():
    t = tune.Table()
    t.add("fwd", 2, 256, 512, tune.Config(128, 128, 2), 1.0)
    try:
        tune.install(t)
        assert tune.pick("fwd", 2, 256, 512) == tune.Config(128, 128, 2)
        assert tune.pick("wgrad", 2, 256, 512) is None
    finally:
        tune.install(None)
    assert tune.pick("fwd", 2, 256, 512) is None


def test_tuned_call_leaves_the_callers_defaults():
    """A config set by the caller (bench --tile-m, say) stays in force around
    a tuned call: the tuned entry travels with the call instead."""
    try:
        _lib.set_tile_config(128, 256, 4)
        _lib.set_schedule(_lib.SCHED_TILES, 0)
        assert tune.call_config(tune.Config(256, 128, 16, _lib.SCHED_SPLIT_TAIL, 3)) == [256, 128, 16, 2, 3]
        assert _lib.current_config() == ((128, 256, 4), (_lib.SCHED_TILES, 0))
    finally:
        _lib.set_tile_config(0, 0, 0)
        _lib.set_schedule(_lib.SCHED_DEFAULT, 0)
