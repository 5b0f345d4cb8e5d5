"""The no-allocation H_res backward keeps its array's device address per CUDA
context (mhc-proj_b200/csrc/context_cache.h): a device reset or another
context on the same device must look the address up again instead of using
one from a module that is gone.  The cache logic is host C++ with no CUDA
dependency; it is compiled here with g++ and driven with a fake lookup."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "mhc-proj_b200", "csrc")


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_address_is_kept_per_context(tmp_path):
    exe = str(tmp_path / "context_cache_check")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", CSRC,
                    os.path.join(HERE, "context_cache_check.cpp"), "-o", exe, "-pthread"], check=True)
    out = subprocess.run([exe], capture_output=True, text=True)
    assert out.returncode == 0 and out.stdout.strip() == "ok", out.stdout + out.stderr
