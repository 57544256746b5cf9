"""ctypes binding of the in-tree C ABI ``libmxgg.so`` (declared in include/mxgg.h).

Loading fails loudly: there is no CPU or Triton fallback anywhere in the
library.  Build the shared object with ``python grouped-gemms_b200/build.py``.
"""

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmxgg.so")
_DEFAULT_LIB_PATH = LIB_PATH
_CSRC = os.path.join(os.path.dirname(_HERE), "csrc")
_HEADER = os.path.join(os.path.dirname(os.path.dirname(_HERE)), "include", "mxgg.h")


def source_files():
    """The files libmxgg.so is compiled from (kernels, C ABI, public header)."""
    return [os.path.join(_CSRC, f) for f in sorted(os.listdir(_CSRC)) if f.endswith((".cu", ".cuh"))] + [_HEADER]


def source_digest():
    """First 16 hex digits of the sha256 over the library's sources (names
    and contents), or None where the sources are not present.  The build
    embeds it (mxgg_build_id), so a library built from other sources is
    refused instead of being called with argument lists it does not take."""
    import hashlib
    if not (os.path.isdir(_CSRC) and os.path.exists(_HEADER)):
        return None
    h = hashlib.sha256()
    for f in source_files():
        h.update(os.path.basename(f).encode() + b"\0")
        with open(f, "rb") as fh:
            h.update(fh.read())
        h.update(b"\0")
    return h.hexdigest()[:16]

MXGG_OK = 0
DTYPE_BF16, DTYPE_F16, DTYPE_F32 = 0, 1, 2
QUANT_ROWS, QUANT_COLS = 0, 1
SCALE_ROW_MAJOR, SCALE_BLOCKED = 0, 1
SCHED_DEFAULT, SCHED_TILES, SCHED_SPLIT_TAIL = 0, 1, 2
FMT_E4M3, FMT_E2M1 = 0, 1



class GemmConfig(ctypes.Structure):
    """``mxgg_gemm_config``: a call's tile and schedule choice (0 = the
    process default, which defaults to the library's heuristic) and the
    layout of the scales it is given (SCALE_ROW_MAJOR or SCALE_BLOCKED)."""
    _fields_ = [("tile_m", ctypes.c_int32), ("tile_n", ctypes.c_int32), ("group_m", ctypes.c_int32),
                ("schedule", ctypes.c_int32), ("split_max", ctypes.c_int32), ("scale_layout", ctypes.c_int32),
                ("reserved", ctypes.c_int32 * 2)]


def gemm_config(cfg, scale_layout: int = SCALE_ROW_MAJOR):
    """A pointer to a GemmConfig for `cfg` -- a (tile_m, tile_n, group_m,
    schedule, split_max) sequence, or None for the process defaults -- and
    `scale_layout`; None when both are defaults."""
    if cfg is None and scale_layout == SCALE_ROW_MAJOR:
        return None
    vals = [int(v) for v in (cfg if cfg is not None else ())]
    vals += [0] * (5 - len(vals))
    return ctypes.pointer(GemmConfig(*vals[:5], int(scale_layout)))


# every symbol include/mxgg.h declares, with (restype, argtypes)
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_int = ctypes.c_int
_cfg = ctypes.POINTER(GemmConfig)
SIGNATURES = {
    "mxgg_grouped_mm_workspace_size": (_i64, [_i64, _i64, _i64, _i64]),
    "mxgg_wgrad_workspace_size": (_i64, [_i64, _i64, _i64, _i64]),
    "mxgg_grouped_mm": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _int, _vp, _i64, _vp]),
    "mxgg_grouped_mm_cfg": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _int, _cfg, _vp, _i64,
                                   _vp]),
    "mxgg_wgrad_cfg": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _int, _cfg, _vp, _i64, _vp]),
    "mxgg_grouped_mm_segments_cfg": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _vp,
                                            _int, _cfg, _vp, _i64, _vp]),
    "mxgg_grouped_mm_mx_cfg": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _vp, _int,
                                      _vp, _vp, _vp, _vp, _cfg, _vp, _i64, _vp]),
    "mxgg_wgrad_accumulate_cfg": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _cfg, _vp, _i64,
                                         _vp]),
    "mxgg_wgrad": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _int, _vp, _i64, _vp]),
    "mxgg_grouped_mm_segments_workspace_size": (_i64, [_i64, _i64, _i64, _i64, _i64]),
    "mxgg_grouped_mm_segments": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _vp, _int,
                                        _vp, _i64, _vp]),
    "mxgg_grouped_mm_mx": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32, _vp, _int, _vp,
                                  _vp, _vp, _vp, _vp, _i64, _vp]),
    "mxgg_grouped_mm_ep": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i32,
                                  ctypes.POINTER(_vp), ctypes.POINTER(_i64), ctypes.POINTER(_vp), _i32, _i32, _vp, _vp,
                                  _i32, _vp, _vp, _i64, _i32, _i64, _vp, _vp, _int, _vp, _i64, _vp]),
    "mxgg_query_tile_m": (_i32, []),
    "mxgg_ep_atom_bytes": (_i64, [_i64, _i64, _i64]),
    "mxgg_pack_a_atoms": (_int, [_vp, _vp, _i64, _i64, _i64, _vp, _vp]),
    "mxgg_pack_a_atoms_multi": (_int, [_vp, _i64, _i32, ctypes.POINTER(_i64), ctypes.POINTER(_i64),
                                       ctypes.POINTER(_vp), ctypes.POINTER(_i64), ctypes.POINTER(_vp), _vp]),
    "mxgg_peer_signal": (_int, [_vp, _i32, _vp]),
    "mxgg_inbox_unpack": (_int, [_vp, _vp, _vp, _i64, _i64, _vp]),
    "mxgg_ipc_alloc": (_int, [_i64, ctypes.POINTER(_vp), ctypes.c_char_p]),
    "mxgg_ipc_free": (_int, [_vp]),
    "mxgg_ipc_open": (_int, [ctypes.c_char_p, ctypes.POINTER(_vp)]),
    "mxgg_ipc_close": (_int, [_vp]),
    "mxgg_copy_async": (_int, [_vp, _vp, _i64, _vp]),
    "mxgg_peer_barrier": (_int, [ctypes.POINTER(_vp), _i32, _i32, _i32, _vp]),
    "mxgg_replica_sum": (_int, [ctypes.POINTER(_vp), _i32, _i32, _i64, _int, _vp]),
    "mxgg_wgrad_accumulate": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _vp, _i64, _vp]),
    "mxgg_grouped_mm_noalloc": (_int, [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _vp, _int, _vp]),
    "mxgg_quantize_mx": (_int, [_vp, _int, _i64, _i64, _vp, _vp, _int, _int, _vp]),
    "mxgg_blocked_scale_bytes": (_i64, [_i64, _i64, _i64]),
    "mxgg_quantize_mx_blocked": (_int, [_vp, _int, _i64, _i64, _vp, _vp, _vp, _i64, _i64, _vp]),
    "mxgg_quantize_mx_fp4": (_int, [_vp, _int, _i64, _i64, _vp, _vp, _int, _vp]),
    "mxgg_quantize_mx_gather": (_int, [_vp, _int, _i64, _vp, _i64, _i64, _vp, _vp, _vp]),
    "mxgg_combine_topk": (_int, [_vp, _i64, _vp, _vp, _i64, _i64, _i32, _vp, _vp]),
    "mxgg_build_tile_map": (_int, [_vp, _i64, _i64, _i32, _vp, _vp]),
    "mxgg_set_tile_config": (_int, [_i32, _i32, _i32]),
    "mxgg_set_schedule": (_int, [_i32, _i32]),
    "mxgg_set_wait_limit": (_int, [_i64]),
    "mxgg_wait_limit": (_i64, []),
    "mxgg_device_status": (_int, [ctypes.POINTER(ctypes.c_uint32), _int, _vp]),
    "mxgg_last_error": (ctypes.c_char_p, []),
    "mxgg_version": (_i32, []),
    "mxgg_build_id": (ctypes.c_char_p, []),
}

_lib = None
_lock = threading.Lock()


class MxggError(RuntimeError):
    pass


def load():
    """Load libmxgg.so (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise MxggError(
                f"mxgg CUDA library not found at {LIB_PATH}; build it with "
                "`python grouped-gemms_b200/build.py` (nvcc, sm_100a)")
        lib = ctypes.CDLL(LIB_PATH)
        if LIB_PATH == _DEFAULT_LIB_PATH:
            want = source_digest()
            lib.mxgg_build_id.restype = ctypes.c_char_p
            got = lib.mxgg_build_id().decode()
            if want is not None and got != want:
                raise MxggError(
                    f"{LIB_PATH} was built from other sources (build id {got}, sources {want}); rebuild it "
                    "with `python grouped-gemms_b200/build.py`")
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def check(rc: int, what: str) -> None:
    if rc != MXGG_OK:
        msg = load().mxgg_last_error().decode(errors="replace")
        raise MxggError(f"{what} failed (code {rc}): {msg}")


def set_wait_limit(ns: int = 0) -> None:
    """Limit of every bounded device-side wait, in ns (0: the default 1 s).
    A wait that runs out sets a device status bit and its kernel returns."""
    check(load().mxgg_set_wait_limit(int(ns)), "mxgg_set_wait_limit")


def wait_limit() -> int:
    """The bounded-wait limit in ns."""
    return int(load().mxgg_wait_limit())


def device_status(clear: bool = True, stream=None) -> int:
    v = ctypes.c_uint32(0)
    check(load().mxgg_device_status(ctypes.byref(v), int(clear), stream), "mxgg_device_status")
    return v.value


# the library's process-wide GEMM config as last set through this module
_config = {"tile": (0, 0, 0), "schedule": (SCHED_DEFAULT, 0)}


def set_tile_config(tile_m: int = 0, tile_n: int = 0, group_m: int = 0) -> None:
    """Tile shape for later GEMM calls (0 = automatic): tile_m 128 (one CTA)
    or 256 (a CTA pair), tile_n 128 or 256, group_m the rasterisation band.
    The setting is process-wide (every thread, every device)."""
    check(load().mxgg_set_tile_config(tile_m, tile_n, group_m), "mxgg_set_tile_config")
    _config["tile"] = (tile_m, tile_n, group_m)


def set_schedule(schedule: int = SCHED_DEFAULT, split_max: int = 0) -> None:
    """Work schedule of later GEMM calls: SCHED_SPLIT_TAIL (default) cuts the
    tiles of the last partial round along the contraction for idle CTA pairs,
    SCHED_TILES deals whole tiles; split_max caps the pieces per tile.
    Process-wide, like set_tile_config."""
    check(load().mxgg_set_schedule(schedule, split_max), "mxgg_set_schedule")
    _config["schedule"] = (schedule, split_max)


def current_config():
    """((tile_m, tile_n, group_m), (schedule, split_max)) as last set here."""
    return _config["tile"], _config["schedule"]
