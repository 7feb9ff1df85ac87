"""Builds the native library in-tree: shorokoo_b200/libshorokoo_b200.so.

C++ sources compile with g++, CUDA sources with nvcc for sm_100a only; the CUDA runtime is linked
statically so the library loads on a machine without a GPU driver (tests that only check loading
and exported symbols run there). Objects go to shorokoo_b200/_build/ and are rebuilt when a source
or header is newer.

    python -m shorokoo_b200.build          # or: python shorokoo_b200/build.py
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libshorokoo_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CXXFLAGS = ["-O2", "-std=c++17", "-fPIC", "-Wall", "-Wno-sign-compare", "-Wno-psabi", "-fvisibility=hidden",
            f"-I{CUDA_HOME}/include", f"-I{INCLUDE}", f"-I{CSRC}"]
NVFLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden",
                  f"-I{INCLUDE}", f"-I{CSRC}", "--expt-relaxed-constexpr"]


def _sources():
    cpp = sorted(glob.glob(os.path.join(CSRC, "*.cpp")))
    cu = sorted(glob.glob(os.path.join(CSRC, "kernels", "*.cu")))
    return cpp, cu


def _headers():
    return (glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "kernels", "*.h")) +
            glob.glob(os.path.join(CSRC, "kernels", "*.cuh")) +
            glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(obj: str, src: str, newest_header: float) -> bool:
    if not os.path.exists(obj):
        return True
    t = os.path.getmtime(obj)
    return t < os.path.getmtime(src) or t < newest_header


def _compile(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("compile failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r.stderr


def build(verbose: bool = False, jobs: int = 0) -> str:
    os.makedirs(BUILD, exist_ok=True)
    cpp, cu = _sources()
    newest = max(os.path.getmtime(h) for h in _headers())
    jobs = jobs or min(16, os.cpu_count() or 4)
    cmds, objs = [], []
    for src in cpp:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if _stale(obj, src, newest):
            cmds.append(["g++"] + CXXFLAGS + ["-c", src, "-o", obj])
    for src in cu:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if _stale(obj, src, newest):
            cmds.append([NVCC] + NVFLAGS + ["-c", src, "-o", obj])
    if cmds:
        with cf.ThreadPoolExecutor(jobs) as ex:
            for err in ex.map(_compile, cmds):
                if verbose and err:
                    sys.stderr.write(err)
    relink = cmds or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)
    if relink:
        vs = os.path.join(BUILD, "exports.map")
        with open(vs, "w") as f:
            f.write("{ global: sb_*; local: *; };\n")
        tmp = LIB + ".tmp"
        _compile([NVCC] + ARCH + ["-shared", "-o", tmp] + objs +
                 ["-cudart", "static", "-Xlinker", f"--version-script={vs}", "-lpthread", "-ldl", "-lrt"])
        shutil.move(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
