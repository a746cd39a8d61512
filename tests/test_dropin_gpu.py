"""The drop-in C++ program (tests/cpp/test_dropin.cu), written against the
reference's header names, built against include/ + libmpk.so and run on the GPU."""
import os
import shutil
import subprocess

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_dropin_program_runs(mpk_lib, cuda, tmp_path):
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    lib_dir = os.path.dirname(mpk_lib.library_path())
    exe = tmp_path / "test_dropin"
    subprocess.run([nvcc, "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a",
                    f"-I{os.path.join(ROOT, 'include')}",
                    os.path.join(ROOT, "tests", "cpp", "test_dropin.cu"), f"-L{lib_dir}", "-lmpk",
                    "-Xlinker", "-rpath", "-Xlinker", lib_dir, "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ALL PASS" in r.stdout
