"""The C ABI from plain C: `include/mxgg.h` compiles as C99 with gcc, a C
program links `libmxgg.so` and calls the entry points that need no GPU
(version, workspace sizes, argument validation and `mxgg_last_error`).  This
is the binding a non-Python host of the reference's path would write."""
import os
import shutil
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "grouped-gemms_b200", "mxgg")

C_SRC = r"""
#include <stdio.h>
#include <string.h>
#include "mxgg.h"

int main(void) {
  int v = mxgg_version();
  int64_t fwd = mxgg_grouped_mm_workspace_size(16640, 8192, 8192, 8);
  int64_t wg = mxgg_wgrad_workspace_size(8192, 8192, 16640, 8);
  int64_t bad = mxgg_grouped_mm_workspace_size(-1, 8, 8, 1);
  int rc = mxgg_set_tile_config(64, 0, 0);
  const char* msg = mxgg_last_error();
  int ok = mxgg_set_tile_config(0, 0, 0);
  printf("%d %lld %lld %lld %d %d %s\n", v, (long long)fwd, (long long)wg, (long long)bad, rc, ok,
         strstr(msg, "tile_m") ? "msg-ok" : msg);
  /* the fused quantised output rejects N % 32 != 0 before touching a GPU */
  char buf[64];
  void* p = (void*)(((uintptr_t)buf + 15) & ~(uintptr_t)15);
  int rq = mxgg_grouped_mm_mx(p, p, p, p, (const int32_t*)p, 0, 64, 48, 64, 1, 1, MXGG_FMT_E4M3, 0,
                              MXGG_DTYPE_BF16, p, p, 0, 0, p, 1 << 20, 0);
  printf("%d %s %s\n", rq, strstr(mxgg_last_error(), "N % 32") ? "mx-ok" : mxgg_last_error(), mxgg_build_id());
  return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_c_program_links_and_calls_the_abi():
    lib = os.path.join(LIBDIR, "libmxgg.so")
    assert os.path.exists(lib), "build the library first (python grouped-gemms_b200/build.py)"
    d = tempfile.mkdtemp(prefix="mxgg_c_")
    try:
        src = os.path.join(d, "t.c")
        exe = os.path.join(d, "t")
        with open(src, "w") as f:
            f.write(C_SRC)
        subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), src, "-o", exe,
                        "-L", LIBDIR, "-lmxgg", "-Wl,-rpath," + LIBDIR], check=True)
        out = subprocess.run([exe], check=True, capture_output=True, text=True).stdout.split()
    finally:
        shutil.rmtree(d, ignore_errors=True)
    v, fwd, wg, bad, rc, ok, msg, rq, mx_msg, build_id = out
    assert int(v) > 0
    assert int(fwd) > 0 and int(wg) > 0
    assert int(bad) == -1
    assert int(rc) == 1 and int(ok) == 0           # MXGG_ERR_INVALID, then MXGG_OK
    assert msg == "msg-ok"
    assert int(rq) == 3 and mx_msg == "mx-ok"                  # MXGG_ERR_UNSUPPORTED
    assert len(build_id) == 16 and build_id != "unversioned"
