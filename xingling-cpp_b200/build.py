"""Build the XingLing B200 engine in-tree.

Outputs (next to this file, git-ignored, shipped with the tree):
  libxl_engine.so                          the C-ABI library (include/xl_engine.h)
  llm_cpp_engine.cpython-*.so              the pybind11 module over it

CUDA sources compile for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``).
The build is incremental (object newer than its sources and headers is kept)
and needs no GPU.  Run ``python build.py`` or call ``build()``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
CXX = os.environ.get("XL_CXX", "g++")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["decode.cu", "decode_persistent.cu", "prefill.cu", "gemm_tc.cu", "engine.cu", "batch.cu", "c_api.cu"]
LIB = os.path.join(HERE, "libxl_engine.so")
EXT = os.path.join(HERE, "llm_cpp_engine" + sysconfig.get_config_var("EXT_SUFFIX"))


def _headers() -> list[str]:
    hs = [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    hs += [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    return hs


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {os.path.basename(cmd[-1])}")
    if os.environ.get("XL_BUILD_VERBOSE"):
        sys.stderr.write(r.stdout + r.stderr)


def _nvcc_obj(src: str, verbose_ptxas: bool) -> str:
    obj = os.path.join(OBJ, os.path.splitext(src)[0] + ".o")
    deps = [os.path.join(CSRC, src)] + _headers()
    if _stale(obj, deps):
        cmd = [NVCC, "-std=c++17", "-O3", *ARCH, "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
               "-I", INCLUDE, "-I", CSRC, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose_ptxas:
            cmd[5:5] = ["-Xptxas", "-v"]
        _run(cmd)
    return obj


def build(verbose_ptxas: bool = False) -> None:
    os.makedirs(OBJ, exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(CU_SOURCES)) as ex:
        objs = list(ex.map(lambda s: _nvcc_obj(s, verbose_ptxas), CU_SOURCES))
    if _stale(LIB, objs):
        _run([NVCC, "-shared", *ARCH, "-o", LIB, *objs, "-lnccl", "-ldl", "-Xlinker", "--no-undefined"])
    import pybind11

    mod_src = os.path.join(CSRC, "pybind_module.cpp")
    if _stale(EXT, [mod_src, LIB] + _headers()):
        cxx = shutil.which(CXX) or "g++"
        _run([cxx, "-std=c++17", "-O2", "-fPIC", "-shared", "-fvisibility=hidden",
              "-I", pybind11.get_include(), "-I", sysconfig.get_paths()["include"], "-I", INCLUDE,
              mod_src, "-o", EXT, "-L", HERE, "-lxl_engine", "-Wl,-rpath,$ORIGIN"])


if __name__ == "__main__":
    build(verbose_ptxas="-v" in sys.argv)
    print(LIB)
    print(EXT)
