"""The C ABI from plain C (no GPU needed): include/lifscan_b200.h compiles as
C11 with warnings as errors, a C program links against liblifb.so, and the
host-side paths behave as the header states (ABI version, workspace sizes,
argument errors reported by status and message, empty problems succeed)."""
import os
import shutil
import subprocess

import pytest

from hard_resets_compose_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

PROGRAM = r"""
#include <stdio.h>
#include <string.h>
#include "lifscan_b200.h"

int main(void)
{
    if (lifb_abi_version() != %(abi)d) return 2;
    if (lifb_scan_fwd_v3_workspace_bytes(1024, 4096, 64, 16) == 0) return 3;
    if (lifb_scan_fwd_v3_workspace_bytes(1024, 4096, 48, 16) != 0) return 4;   /* T %% C != 0 */
    if (lifb_scan_bwd_workspace_bytes(1024, 4096, 64) == 0) return 5;
    if (lifb_serial_fwd(NULL, NULL, NULL, NULL, -1, 4, 0.9f, 1.0f, 0.0f, NULL) != LIFB_ERR_INVALID_ARGUMENT)
        return 6;
    if (strstr(lifb_last_error(), "negative") == NULL) return 7;
    /* T not a multiple of C: refused before any CUDA call */
    float *fake = (float *)(size_t)256;
    if (lifb_scan_fwd_v3(fake, fake, fake, fake, 100, 8, 0.9f, 1.0f, 0.0f, 64, 16, -1, NULL, 0, NULL, NULL) !=
        LIFB_ERR_INVALID_ARGUMENT)
        return 8;
    if (lifb_serial_fwd(NULL, NULL, NULL, NULL, 0, 16, 0.9f, 1.0f, 0.0f, NULL) != LIFB_OK) return 9;
    printf("ok %%s\n", lifb_status_string(LIFB_ERR_WORKSPACE));
    return 0;
}
"""


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc is not installed")
def test_header_compiles_as_c_and_links(tmp_path):
    lib = _lib.load()  # builds the library if needed
    libdir = os.path.dirname(_lib._build.LIB)
    src = tmp_path / "abi.c"
    src.write_text(PROGRAM % {"abi": _lib.ABI_VERSION})
    exe = tmp_path / "abi"
    cmd = ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
           "-o", str(exe), "-L", libdir, "-llifb", f"-Wl,-rpath,{libdir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    assert r.stdout.startswith("ok ") and lib.lifb_status_string(3).decode() in r.stdout


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc is not installed")
def test_c_example_compiles_and_links(tmp_path):
    """The C caller of the library (tests/c/lif_example.c) compiles with
    warnings as errors and links against liblifb.so and the CUDA runtime
    (running it needs a GPU)."""
    _lib.load()
    libdir = os.path.dirname(_lib._build.LIB)
    src = os.path.join(ROOT, "tests", "c", "lif_example.c")
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cmd = ["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
           "-I", os.path.join(cuda, "include"), src, "-o", str(tmp_path / "lif"), "-L", libdir, "-llifb",
           "-L", os.path.join(cuda, "lib64"), "-lcudart", f"-Wl,-rpath,{libdir}"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
