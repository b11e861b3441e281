"""include/gs200.h is a plain C header: a C99 program (as a cgo / FFI user would write) and
a C++ program include it, link against libgs200.so and run host-only calls -- the
version string and an argument error that returns before any device work -- without a
GPU."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "gsplat_tt_b200")

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "gs200.h"

int main(void) {
    const char* v = gs_version();
    if (strncmp(v, "gs200", 5) != 0) return 2;
    /* a negative pair count is rejected on the host, before any device call */
    gs_status s = gs_sort_pairs(NULL, NULL, -1, 45, NULL, NULL, NULL, 0, NULL);
    if (s != GS_ERR_ARG) return 3;
    if (strstr(gs_last_error(), "n must be") == NULL) return 4;
    printf("ok %s\n", v);
    return 0;
}
"""


@pytest.mark.parametrize("compiler,std,ext", [("gcc", "-std=c99", "c"), ("g++", "-std=c++17", "cpp")])
def test_header_compiles_links_and_runs(tmp_path, compiler, std, ext):
    if shutil.which(compiler) is None:
        pytest.skip(f"{compiler} not installed")
    if not os.path.exists(os.path.join(LIBDIR, "libgs200.so")):
        pytest.fail("libgs200.so is not built (python -m gsplat_tt_b200.build)")
    src = tmp_path / f"main.{ext}"
    src.write_text(PROGRAM)
    exe = tmp_path / "main"
    subprocess.run([compiler, std, "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    str(src), "-L", LIBDIR, "-lgs200", f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)],
                   check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, (out.returncode, out.stderr)
    assert out.stdout.startswith("ok gs200")
