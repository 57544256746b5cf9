"""Autotune harness host logic (no GPU): the candidate space, applying and
restoring a config through the C ABI, best-config selection, dealing points
to GPUs, and the table's JSON round trip, merge and lookup."""
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


def test_applied_sets_then_restores(monkeypatch):
    calls = []
    monkeypatch.setattr(_lib, "set_tile_config", lambda *a: calls.append(("tile",) + a))
    monkeypatch.setattr(_lib, "set_schedule", lambda *a: calls.append(("sched",) + a))
    cfg = tune.Config(128, 256, 4, _lib.SCHED_TILES, 0)
    with tune.applied(cfg):
        assert calls == [("tile", 128, 256, 4), ("sched", _lib.SCHED_TILES, 0)]
    assert calls[2:] == [("tile", 0, 0, 0), ("sched", _lib.SCHED_DEFAULT, 0)]
    calls.clear()
    with tune.applied(None):
        pass
    assert calls == []
    with pytest.raises(ValueError):
        with tune.applied(tune.Config(tile_n=64)):
            pass


def test_applied_restores_after_an_error(monkeypatch):
    calls = []
    monkeypatch.setattr(_lib, "set_tile_config", lambda *a: calls.append(a))
    monkeypatch.setattr(_lib, "set_schedule", lambda *a: None)
    with pytest.raises(RuntimeError):
        with tune.applied(tune.Config(256, 128, 8)):
            raise RuntimeError("call failed")
    assert calls[-1] == (0, 0, 0)


def test_applied_through_the_real_library():
    # the setters need no GPU; an out-of-range value is rejected by the library
    with tune.applied(tune.Config(128, 128, 2, _lib.SCHED_TILES, 0)):
        pass
    with pytest.raises(_lib.MxggError):
        _lib.set_tile_config(64, 0, 0)
    _lib.set_tile_config(0, 0, 0)


def test_tune_point_picks_the_fastest_and_skips_rejected(monkeypatch):
    monkeypatch.setattr(_lib, "set_tile_config", lambda *a: None)
    monkeypatch.setattr(_lib, "set_schedule", lambda *a: None)
    cfgs = tune.config_space()[:5]
    fake = {cfgs[0]: 3.0, cfgs[1]: 1.0, cfgs[2]: 1.0, cfgs[4]: 2.0}
    current = {}

    def timer(run):
        c = current["cfg"]
        if c not in fake:
            raise _lib.MxggError("rejected")
        return fake[c]

    orig = tune.applied

    def spy(cfg):
        current["cfg"] = cfg
        return orig(cfg)

    monkeypatch.setattr(tune, "applied", spy)
    times = tune.tune_point(lambda: None, cfgs, timer)
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


def test_applied_restores_the_callers_config():
    """A config set by the caller (bench --tile-m, say) comes back after a
    tuned call, not the library default."""
    try:
        _lib.set_tile_config(128, 256, 4)
        _lib.set_schedule(_lib.SCHED_TILES, 0)
        with tune.applied(tune.Config(256, 128, 16, _lib.SCHED_SPLIT_TAIL, 3)):
            assert _lib.current_config() == ((256, 128, 16), (_lib.SCHED_SPLIT_TAIL, 3))
        assert _lib.current_config() == ((128, 256, 4), (_lib.SCHED_TILES, 0))
    finally:
        _lib.set_tile_config(0, 0, 0)
        _lib.set_schedule(_lib.SCHED_DEFAULT, 0)
