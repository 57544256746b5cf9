"""Autotuning harness for the sm_100a grouped GEMM.

This replaces the reference's Triton tuning pair (``tune_driver.py``, which
shards (E, N, K) points over GPUs, and ``tune_worker.py``, which times the
candidate configs of one point, ``tune_worker.py:87-91``) and the table it
fills (``_BEST_CFGS``, which ``_pick_config`` looks up, ``forward.py:399-459``).
The knobs here are the B200 kernel's own:

* tile rows ``tile_m``: 256 is a CTA pair (``cta_group::2``), 128 is one CTA;
* tile columns ``tile_n``: 128 or 256;
* ``group_m``: the rasterisation band, in row tiles;
* the work schedule: whole tiles, or a split of the last round's tiles;
* ``split_max``: the most pieces a split tile is cut into.

One process per GPU.  Points are dealt round-robin, every worker writes its
own partial table, and the parent merges them: there is no collective, so one
GPU failing does not stall the others.  Each candidate is timed with CUDA
events on the launching stream, after warm-up, with L2 flushed before every
timed launch.

A table is JSON: ``{"device": ..., "entries": [{"pass": "fwd", "E": 8,
"N": 2048, "K": 5120, "M": 16640, "config": {...}, "us": 123.4}, ...]}``,
keyed on the call: ("fwd", E, N, K) for ``triton_mxfp8_grouped_mm`` with
weight (E, N, K) -- dgrad included, as the forward call with N and K swapped
-- and ("wgrad", E, N, K) for ``triton_mxfp8_wgrad`` with output (E, N, K).
``install(table)`` makes those entry points look up their call and pass the
entry's config with the call itself (``mxgg_gemm_config``): no process-wide
setting changes, so threads issuing differently tuned GEMMs do not race.

At import the package installs its own table, ``tables/b200_llama4.json``:
the 36 Llama4 sweep shapes x {fwd, wgrad} (dgrad shapes are among the
forward ones), tuned on a B200 at M = 16640.  The environment variable
``MXGG_TUNE_TABLE`` names another table to install instead, or, set to
``none``, installs none.  Without an entry for a call, the library's own
heuristic applies.

    python -m mxgg.tune --shapes 0,4,8 --passes fwd,wgrad --gpus 8 --out table.json
"""

import argparse
import json
import os
import tempfile
from dataclasses import asdict, dataclass
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple

from . import _lib

M_TOKENS = 16640
PASSES = ("fwd", "dgrad", "wgrad")


def llama4_shapes() -> List[Tuple[int, int, int, int]]:
    """The 36 (E, M, N, K) points of the reference's sweep, in its order (bench.py:113-122)."""
    return [(e, M_TOKENS, n, k) for e in (1, 2, 4, 8) for n in (2048, 5120, 8192) for k in (2048, 5120, 8192)]


@dataclass(frozen=True)
class Config:
    """One kernel configuration.  Zero means the library's automatic choice."""
    tile_m: int = 0
    tile_n: int = 0
    group_m: int = 0
    schedule: int = _lib.SCHED_DEFAULT
    split_max: int = 0

    def as_list(self) -> List[int]:
        """The fields in ``mxgg_gemm_config`` order."""
        return [self.tile_m, self.tile_n, self.group_m, self.schedule, self.split_max]

    def valid(self) -> bool:
        return (self.tile_m in (0, 128, 256) and self.tile_n in (0, 128, 256) and self.group_m >= 0
                and self.schedule in (_lib.SCHED_DEFAULT, _lib.SCHED_TILES, _lib.SCHED_SPLIT_TAIL)
                and (self.split_max == 0 or 2 <= self.split_max <= 64))


DEFAULT = Config()


def config_space(tile_ms: Sequence[int] = (256, 128), tile_ns: Sequence[int] = (256, 128),
                 schedules: Sequence[int] = (_lib.SCHED_SPLIT_TAIL, _lib.SCHED_TILES)) -> List[Config]:
    """Candidate configs: every tile shape, each with raster bands suited to
    it (wide for a CTA pair, narrow for one CTA), and each schedule."""
    out = []
    for tm in tile_ms:
        bands = (8, 16, 32) if tm == 256 else (2, 4, 8)
        for tn in tile_ns:
            for g in bands:
                for sch in schedules:
                    out.append(Config(tm, tn, g, sch, 0))
    return out


def call_config(cfg: Optional[Config]) -> Optional[List[int]]:
    """The per-call config argument of the mxgg ops for `cfg` (None: the
    process defaults).  Nothing process-wide is changed: the library takes the
    config with the call (``mxgg_gemm_config``)."""
    if cfg is None:
        return None
    if not cfg.valid():
        raise ValueError(f"invalid config {cfg}")
    return cfg.as_list()


# ------------------------------------------------------------------ tables
Key = Tuple[str, int, int, int]


class Table:
    """Best config per (pass, E, N, K), with its time."""

    def __init__(self, device: str = "", entries: Optional[Dict[Key, Tuple[Config, float, int]]] = None):
        self.device = device
        self.entries: Dict[Key, Tuple[Config, float, int]] = dict(entries or {})

    def add(self, pass_: str, E: int, N: int, K: int, cfg: Config, us: float, M: int = M_TOKENS) -> None:
        key = (pass_, E, N, K)
        old = self.entries.get(key)
        if old is None or us < old[1]:
            self.entries[key] = (cfg, us, M)

    def lookup(self, pass_: str, E: int, N: int, K: int) -> Optional[Config]:
        e = self.entries.get((pass_, E, N, K))
        return e[0] if e else None

    def merge(self, other: "Table") -> "Table":
        for (p, E, N, K), (cfg, us, M) in other.entries.items():
            self.add(p, E, N, K, cfg, us, M)
        if not self.device:
            self.device = other.device
        return self

    def to_json(self) -> dict:
        rows = [{"pass": p, "E": E, "N": N, "K": K, "M": M, "config": asdict(cfg), "us": round(us, 2)}
                for (p, E, N, K), (cfg, us, M) in sorted(self.entries.items())]
        return {"device": self.device, "entries": rows}

    @classmethod
    def from_json(cls, d: dict) -> "Table":
        t = cls(d.get("device", ""))
        for r in d.get("entries", []):
            cfg = Config(**r["config"])
            if not cfg.valid():
                raise ValueError(f"invalid config in table: {r['config']}")
            t.add(r["pass"], int(r["E"]), int(r["N"]), int(r["K"]), cfg, float(r["us"]), int(r.get("M", M_TOKENS)))
        return t

    def save(self, path: str) -> None:
        tmp = path + ".tmp"
        with open(tmp, "w") as f:
            json.dump(self.to_json(), f, indent=1)
        os.replace(tmp, path)

    @classmethod
    def load(cls, path: str) -> "Table":
        with open(path) as f:
            return cls.from_json(json.load(f))


_installed: Optional[Table] = None


def install(table) -> None:
    """Make the entry points use `table` (a Table, a path, or None to stop)."""
    global _installed
    _installed = Table.load(table) if isinstance(table, str) else table


def pick(pass_: str, E: int, N: int, K: int) -> Optional[Config]:
    """The installed table's config for this point, or None (library default)."""
    return _installed.lookup(pass_, E, N, K) if _installed is not None else None


DEFAULT_TABLE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tables", "b200_llama4.json")


def install_default() -> None:
    """The import-time choice: ``MXGG_TUNE_TABLE`` (a path, or ``none``), else
    the packaged B200 table."""
    env = os.environ.get("MXGG_TUNE_TABLE")
    if env is None:
        install(DEFAULT_TABLE if os.path.exists(DEFAULT_TABLE) else None)
    elif env.strip().lower() in ("", "none", "off", "0"):
        install(None)
    else:
        install(env)


install_default()


# ------------------------------------------------------------------ timing
def call_points(shapes: Sequence[Tuple[int, int, int, int]], passes: Sequence[str]) -> list:
    """Distinct call shapes of the sweep points.  A table is keyed on the
    call, not on the pass: dgrad of point (E, N, K) is the forward call with
    N and K swapped, the same GEMM, so it is tuned (and looked up) as
    ("fwd", E, K, N)."""
    out = []
    for (E, M, N, K) in shapes:
        for p in passes:
            if p not in PASSES:
                raise ValueError(f"unknown pass {p}")
            pt = ("fwd", E, M, K, N) if p == "dgrad" else (p, E, M, N, K)
            if pt not in out:
                out.append(pt)
    return out


def shard(points: Sequence, rank: int, world: int) -> list:
    """This worker's share of the points (round-robin, like the reference's
    driver deals points to GPUs)."""
    return list(points[rank::world])


def best(times: Dict[Config, float]) -> Tuple[Config, float]:
    """The fastest config; ties go to the one tried first."""
    cfg = min(times, key=lambda c: times[c])
    return cfg, times[cfg]


MARGIN = 0.03   # a tuned entry must beat the library's own choice by this much


def worth_keeping(times: Dict[Config, float], confirm: Optional[Callable[[Config], Tuple[float, float]]] = None,
                  margin: float = MARGIN) -> Optional[Tuple[Config, float]]:
    """The fastest config if it beats DEFAULT (the library's own choice, timed
    among the candidates) by `margin`, and -- with `confirm`, which re-times
    (best, DEFAULT) -- still does on a second measurement; else None: the
    call shape keeps the library's choice, so timing noise never installs a
    config that is not really faster."""
    if DEFAULT not in times:
        return best(times)
    cfg, t = best(times)
    if cfg == DEFAULT or t > times[DEFAULT] * (1.0 - margin):
        return None
    if confirm is not None:
        t2, d2 = confirm(cfg)
        if t2 > d2 * (1.0 - margin):
            return None
        t = min(t, t2)
    return cfg, t


def tune_point(run: Callable[[Optional[List[int]]], object], configs: Iterable[Config],
               timer: Callable[[Callable[[], object]], float]) -> Dict[Config, float]:
    """Seconds per call of `run(config)` under each config, the config passed
    with the call (a config the library rejects is skipped)."""
    out: Dict[Config, float] = {}
    for cfg in configs:
        c = call_config(cfg)
        try:
            out[cfg] = timer(lambda: run(c))
        except _lib.MxggError:
            continue
    return out


def cuda_timer(reps: int = 10, warmup: int = 3, flush_bytes: int = 512 << 20):
    """Mean device time of `run`: CUDA events on the current stream around
    each call, a memset larger than L2 before each."""
    import torch
    scratch = torch.empty(flush_bytes, dtype=torch.uint8, device="cuda")

    def timer(run):
        for _ in range(warmup):
            scratch.zero_()
            run()
        total = 0.0
        for _ in range(reps):
            scratch.zero_()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            run()
            e.record()
            e.synchronize()
            total += s.elapsed_time(e)
        if _lib.device_status(clear=True) != 0:
            raise _lib.MxggError("a device-side wait timed out while tuning")
        return total / reps * 1e-3

    return timer


def build_point(pass_: str, E: int, M: int, N: int, K: int, seed: int = 123):
    """Quantised operands of one call shape ("fwd": out (M, N) over K;
    "wgrad": out (E, N, K) over M tokens), offsets as the reference draws them
    (utils.generate_jagged_offs, multiples of 32), and the call to time as a
    function of its config."""
    import random

    import torch

    import utils

    from . import ops
    random.seed(seed + E)
    g = torch.Generator(device="cuda").manual_seed(seed)
    offs = utils.generate_jagged_offs(E, M, multiple_of=32, device="cuda")
    if pass_ == "fwd":
        a_s, a_q = utils.to_mx(torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g))
        b_s, b_q = utils.to_mx(torch.randn(E, N, K, device="cuda", dtype=torch.bfloat16, generator=g))
        return lambda cfg: ops.grouped_mm(a_q, b_q, a_s, b_s, offs, torch.bfloat16, cfg)
    if pass_ == "wgrad":
        go_s, go_q = utils.to_mx_dim1(torch.randn(M, N, device="cuda", dtype=torch.bfloat16, generator=g))
        ia_s, ia_q = utils.to_mx_dim1(torch.randn(M, K, device="cuda", dtype=torch.bfloat16, generator=g))
        return lambda cfg: ops.wgrad(go_q, go_s, ia_q, ia_s, offs, torch.bfloat16, cfg)
    raise ValueError(f"unknown pass {pass_}")


def _worker(rank: int, world: int, points: list, configs: List[Config], reps: int, out_dir: str) -> None:
    """One GPU: time every config on this rank's points, save a partial table."""
    import torch
    torch.cuda.set_device(rank)
    timer = cuda_timer(reps=reps)
    table = Table(torch.cuda.get_device_name(rank))
    for (pass_, E, M, N, K) in shard(points, rank, world):
        run = build_point(pass_, E, M, N, K)
        times = tune_point(run, [DEFAULT] + [c for c in configs if c != DEFAULT], timer)
        confirm = lambda c: (timer(lambda: run(call_config(c))), timer(lambda: run(None)))  # noqa: E731
        kept = worth_keeping(times, confirm) if times else None
        if kept:
            table.add(pass_, E, N, K, kept[0], kept[1] * 1e6, M)
        del run
        torch.cuda.empty_cache()
    table.save(os.path.join(out_dir, f"part{rank}.json"))


def tune(shapes: Sequence[Tuple[int, int, int, int]], passes: Sequence[str] = PASSES,
         configs: Optional[List[Config]] = None, gpus: int = 1, reps: int = 10) -> Table:
    """Tune every (pass, shape) point on `gpus` GPUs (one spawned process per
    GPU, or this process for one) and return the merged table."""
    configs = list(configs or config_space())
    points = call_points(shapes, passes)
    out_dir = tempfile.mkdtemp(prefix="mxgg_tune_")
    if gpus <= 1:
        _worker(0, 1, points, configs, reps, out_dir)
    else:
        import torch.multiprocessing as mp
        mp.start_processes(_worker, args=(gpus, points, configs, reps, out_dir), nprocs=gpus, join=True,
                           start_method="spawn")
    table = Table()
    for r in range(max(gpus, 1)):
        path = os.path.join(out_dir, f"part{r}.json")
        if os.path.exists(path):
            table.merge(Table.load(path))
            os.remove(path)
    os.rmdir(out_dir)
    return table


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--shapes", default="all", help="'all' or comma list of sweep indices 0..35")
    ap.add_argument("--passes", default=",".join(PASSES))
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--reps", type=int, default=10)
    ap.add_argument("--tiles", default="256x256,256x128,128x256,128x128", help="candidate tile_m x tile_n")
    ap.add_argument("--out", required=True)
    a = ap.parse_args(argv)
    shapes = llama4_shapes()
    if a.shapes != "all":
        shapes = [shapes[int(i)] for i in a.shapes.split(",")]
    tiles = [tuple(int(v) for v in t.split("x")) for t in a.tiles.split(",")]
    configs = [c for c in config_space() if (c.tile_m, c.tile_n) in tiles]
    table = tune(shapes, a.passes.split(","), configs, a.gpus, a.reps)
    table.save(a.out)
    for r in table.to_json()["entries"]:
        print(json.dumps(r))


if __name__ == "__main__":
    main()
