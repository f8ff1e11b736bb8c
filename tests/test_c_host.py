"""include/h3b.h is a plain C header: a C program compiles against it, links
libh3b.so and gets the documented error behaviour (CPU only, no device call)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "minimax-h3-multi-dgx-spark_b200", "h3b")


@pytest.mark.skipif(shutil.which("gcc") is None, reason="needs gcc")
def test_c_host_binds_the_abi(tmp_path):
    exe = tmp_path / "abi_smoke"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c_host", "abi_smoke.c"), "-L", LIBDIR, "-lh3b",
                    f"-Wl,-rpath,{LIBDIR}", "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "abi 2" in r.stdout and "rc -1" in r.stdout
