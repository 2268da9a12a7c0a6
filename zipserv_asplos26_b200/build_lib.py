"""Build libzipserv_b200.so (sm_100a) in-tree with nvcc / g++.

The library is the product: CUDA kernels, the reference's C++ ABI
(include/L_API.cuh) and the plain C ABI (include/zipserv_b200.h). The build is
incremental (objects are rebuilt when a source or header is newer).
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIBDIR = os.path.join(PKG, "lib")
OBJDIR = os.path.join(LIBDIR, "obj")
LIB = os.path.join(LIBDIR, "libzipserv_b200.so")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]

NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fopenmp",
                     "--expt-relaxed-constexpr", "-Xptxas", "-v,-warn-spills", f"-I{INCLUDE}", f"-I{CSRC}"]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-fopenmp", f"-I{INCLUDE}", f"-I{CSRC}", f"-I{CUDA}/include"]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h")) + glob.glob(os.path.join(INCLUDE, "*.cuh"))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
    if not _stale(obj, [src] + _headers()):
        return obj
    if src.endswith(".cu"):
        cmd = [NVCC] + NVCC_FLAGS + ["-c", src, "-o", obj]
    else:
        cmd = ["g++"] + CXX_FLAGS + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    log = os.path.join(OBJDIR, os.path.basename(src) + ".log")
    with open(log, "w") as f:
        f.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
    if r.returncode != 0:
        raise RuntimeError(f"compile failed: {src}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"[zipserv build] {os.path.basename(src)}")
    return obj


def build(verbose: bool = False) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    if _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [NVCC] + ARCH + ["-shared", "-o", tmp] + objs + ["-lgomp"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
        if verbose:
            print(f"[zipserv build] linked {LIB}")
    return LIB


if __name__ == "__main__":
    build(verbose=True)
