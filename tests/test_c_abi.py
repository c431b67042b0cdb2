"""The boundary is a plain C ABI: include/dspine_b200.h compiles as pedantic C99 with no CUDA
header, and a C program links libdspine_b200.so and calls it (host validation only, no GPU)."""

import os
import shutil
import subprocess

import pytest

from dspine_b200 import _lib, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

C_PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "dspine_b200.h"

int main(void) {
    size_t ws = 0;
    if (strncmp(dsv_version(), "dspine_b200", 11) != 0) return 1;
    if (strcmp(dsv_status_string(6), "workspace too small") != 0) return 2;
    if (dsv_verify_workspace_size(64, &ws) != 0 || ws == 0) return 3;
    /* refused before any launch: k not a power of two, null pointers, empty batch */
    if (dsv_topk_ids(2, 4096, 4096, 0, NULL, 3, NULL, NULL) != 1) return 4;
    if (dsv_topk_ranked(2, 4096, 4096, 0, NULL, 16, NULL, NULL) != 3) return 5;
    if (dsv_fp8_quantize_rows(0, 64, 64, 0, NULL, NULL, 64, NULL, NULL) != 0) return 6;
    printf("ok %s\n", dsv_version());
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_header_is_c99_and_library_links_from_c(tmp_path):
    build.build()
    src = tmp_path / "abi.c"
    src.write_text(C_PROGRAM)
    exe = tmp_path / "abi"
    libdir = str(_lib.LIB_PATH.parent)
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror",
                    "-I", os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                    "-L", libdir, "-ldspine_b200", "-Wl,-rpath," + libdir], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert out.returncode == 0, (out.returncode, out.stderr)
    assert out.stdout.startswith("ok dspine_b200")
