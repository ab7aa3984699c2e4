"""In-tree build of the sm_100a indexer library and its torch binding.

Produces, next to the Python package (so the files travel with the tree):
  hcu_ops/libhcu_indexer.so   C ABI (include/hcu_indexer.h), nvcc -gencode sm_100a
  hcu_ops/_C<ext-suffix>      pybind11 torch extension over that ABI (g++)
Object files go to _build/.  A target is rebuilt only when a source or header
is newer than it.  Usage: python build.py [--force] [-j N]
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
PKG = os.path.join(HERE, "hcu_ops")
OBJ = os.path.join(HERE, "_build")
INCLUDE = os.path.join(REPO, "include")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")

CU_SOURCES = ["capi.cu", "dequant.cu", "topk.cu", "logits.cu", "mla_kv.cu", "fused.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-Xptxas", "-v"] + ARCH
LIB = os.path.join(PKG, "libhcu_indexer.so")
EXT = os.path.join(PKG, "_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(INCLUDE, "hcu_indexer.h")]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, log=None):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if log is not None:
        with open(log, "w") as f:
            f.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {os.path.basename(cmd[-1])}")
    return r


def build_lib(force=False, jobs=8):
    os.makedirs(OBJ, exist_ok=True)
    hdrs = _headers()
    objs = []
    todo = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(OBJ, src + ".o")
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            todo.append((s, o))

    def compile_one(so):
        s, o = so
        _run([NVCC] + NVCC_FLAGS + ["-I", INCLUDE, "-c", s, "-o", o], log=o + ".log")

    with ThreadPoolExecutor(max_workers=jobs) as ex:
        list(ex.map(compile_one, todo))
    if force or todo or _stale(LIB, objs):
        _run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart_static", "-ldl", "-lrt", "-lpthread"])
    return LIB


def build_ext(force=False):
    import torch.utils.cpp_extension as ce

    src = os.path.join(CSRC, "bind.cpp")
    if not (force or _stale(EXT, [src, LIB, os.path.join(INCLUDE, "hcu_indexer.h")])):
        return EXT
    inc = ce.include_paths() + [sysconfig.get_paths()["include"], os.path.join(CUDA_HOME, "include"), INCLUDE]
    libdirs = ce.library_paths()
    import torch

    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C", "-DTORCH_API_INCLUDE_EXTENSION_H",
           src, "-o", EXT]
    for i in inc:
        cmd += ["-I", i]
    for d in libdirs:
        cmd += ["-L", d, f"-Wl,-rpath,{d}"]
    cmd += ["-L", PKG, "-l:libhcu_indexer.so", "-Wl,-rpath,$ORIGIN",
            "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda"]
    _run(cmd, log=os.path.join(OBJ, "bind.log"))
    return EXT


def build(force=False, jobs=8):
    build_lib(force, jobs)
    build_ext(force)
    return LIB, EXT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=8)
    a = ap.parse_args()
    print(build(a.force, a.j))
