"""The C ABI from plain C: tests/c_client/abi_client.c is compiled with gcc
against include/nvfp4_b200.h, linked against the built library and run (no GPU
needed: it exercises only argument validation)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("gcc") is None, reason="gcc not available")
def test_c_client_builds_and_runs(pkg, tmp_path):
    lib = pkg._lib.LIB_PATH
    exe = tmp_path / "abi_client"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Werror", "-O1",
                    "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "c_client", "abi_client.c"),
                    "-L", os.path.dirname(lib), "-lnvfp4_b200", "-Wl,-rpath," + os.path.dirname(lib),
                    "-o", str(exe)], check=True, capture_output=True, text=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "all passed" in out.stdout
