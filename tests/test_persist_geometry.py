"""The persistent decode kernel's work geometry, checked on the host: the
helpers of xl_kernels.h (box widths for K multiples of 64, and the partial-sum
slots of the split projections, including grids with more CTAs than boxes)
compiled with g++ into tests/persist_geometry_check.cpp and run for every
width up to 4096 and several grid sizes."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA_INC = "/usr/local/cuda/include"


@pytest.mark.skipif(shutil.which("g++") is None or not os.path.isdir(CUDA_INC), reason="needs g++ and CUDA headers")
def test_persist_geometry(tmp_path):
    exe = tmp_path / "geometry"
    subprocess.run(["g++", "-std=c++17", "-O2", f"-I{CUDA_INC}", "-I", os.path.join(ROOT, "xingling-cpp_b200", "csrc"),
                    os.path.join(ROOT, "tests", "persist_geometry_check.cpp"), "-o", str(exe)], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and r.stdout.strip() == "ok", r.stdout + r.stderr
