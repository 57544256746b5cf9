"""Build the in-tree CUDA library ``mxgg/libmxgg.so`` for sm_100a.

    python grouped-gemms_b200/build.py [--force]

nvcc cross-compiles without a GPU.  The shared library lands next to the
Python package that loads it, so it travels with a copy of the source tree.
"""

import argparse
import ctypes
import os
import shutil
import subprocess
import sys
import tempfile
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from mxgg._lib import source_digest, source_files  # noqa: E402
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "mxgg", "libmxgg.so")
ROOT = os.path.dirname(HERE)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
]


def units():
    """The translation units: the C ABI and one per GEMM kernel build
    (compiled in parallel, then linked into one shared library)."""
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith(".cu")]


def built_id(path: str) -> str:
    """The source digest a built library carries ('' if it has none)."""
    try:
        lib = ctypes.CDLL(path)
        fn = lib.mxgg_build_id
    except (OSError, AttributeError):
        return ""
    fn.restype = ctypes.c_char_p
    return fn().decode()


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    if not all(os.path.getmtime(s) <= t for s in source_files() + [__file__]):
        return False
    return built_id(OUT) == source_digest()


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return OUT
    nvcc = os.environ.get("NVCC", "nvcc")
    tmp = tempfile.mkdtemp(prefix="mxgg_build_")
    try:
        def compile_one(src):
            obj = os.path.join(tmp, os.path.basename(src) + ".o")
            cmd = [nvcc, *NVCC_FLAGS, f'-DMXGG_BUILD_ID="{source_digest()}"', "-c", "-o", obj, src]
            if verbose:
                print(" ".join(cmd), flush=True)
            # each nvcc its own scratch directory: parallel runs must not share temporaries
            env = dict(os.environ, TMPDIR=tempfile.mkdtemp(dir=tmp))
            subprocess.run(cmd, check=True, env=env)
            return obj
        srcs = units()
        with ThreadPoolExecutor(max_workers=min(len(srcs), os.cpu_count() or 1)) as ex:
            objs = list(ex.map(compile_one, srcs))
        # only the C ABI is exported: internal symbols stay local to this copy
        cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
               "-Xlinker", "--version-script=" + os.path.join(CSRC, "exports.map"), "-o", OUT + ".tmp", *objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(OUT + ".tmp", OUT)
    finally:
        shutil.rmtree(tmp, ignore_errors=True)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=True))
    sys.exit(0)
