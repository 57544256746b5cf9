"""Build the in-tree CUDA library ``mxgg/libmxgg.so`` for sm_100a.

    python grouped-gemms_b200/build.py [--force]

nvcc cross-compiles without a GPU.  The shared library lands next to the
Python package that loads it, so it travels with a copy of the source tree.
"""

import argparse
import ctypes
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from mxgg._lib import source_digest, source_files  # noqa: E402
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "mxgg", "libmxgg.so")
ROOT = os.path.dirname(HERE)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


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
    cmd = [nvcc, *NVCC_FLAGS, f'-DMXGG_BUILD_ID="{source_digest()}"', "-o", OUT + ".tmp",
           os.path.join(CSRC, "capi.cu")]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(OUT + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=True))
    sys.exit(0)
