"""The C ABI from a C host: tests/capi_host.c is compiled with gcc against
include/bitdance_b200.h, linked to bitdance_b200/libbitdance_b200.so and run. It makes only the
calls that need no GPU (version, status text, workspace sizing, argument checks), so it runs on
CPU. The executable goes to tests/_build/ (ignored by git)."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_c_host_links_and_calls_the_library():
    from bitdance_b200 import build
    lib = build.build_library()
    out_dir = os.path.join(ROOT, "tests", "_build")
    os.makedirs(out_dir, exist_ok=True)
    exe = os.path.join(out_dir, "capi_host")
    libdir = os.path.dirname(lib)
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "tests", "capi_host.c"), "-L", libdir,
                        "-lbitdance_b200", f"-Wl,-rpath,{libdir}", "-o", exe],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    run = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert run.returncode == 0, run.stdout + run.stderr
    assert run.stdout.strip().endswith("ok")
