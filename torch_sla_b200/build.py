"""Build libsla_b200.so (sm_100a) in-tree with nvcc.

The library is a plain C-ABI shared object (``include/sla_b200.h``); it links
NCCL from the nvidia-nccl wheel that PyTorch itself loads, so the row-sharded
solvers share the communicator library already in the process.

Usage: ``python -m torch_sla_b200.build`` (or ``build()`` from Python).
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
BUILD_DIR = os.path.join(REPO_DIR, "_build")
LIB_PATH = os.path.join(PKG_DIR, "libsla_b200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", "-Xptxas", "-O3"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolchain is required")
    return cand


def nccl_paths() -> tuple[str, str]:
    """(include dir, lib dir) of the NCCL that PyTorch loads."""
    try:
        import nvidia.nccl as _n  # type: ignore
        base = list(_n.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    except Exception:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_mtime() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    paths.append(os.path.join(INCLUDE, "sla_b200.h"))
    return max(os.path.getmtime(p) for p in paths)


def build(force: bool = False, verbose: bool = False) -> str:
    nvcc = _nvcc()
    inc, lib = nccl_paths()
    os.makedirs(BUILD_DIR, exist_ok=True)
    hdr_t = _headers_mtime()
    jobs = []
    objs = []
    for src in _sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        stale = force or not os.path.exists(obj) or \
            os.path.getmtime(obj) < max(os.path.getmtime(src), hdr_t)
        if stale:
            cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", INCLUDE, "-I", inc,
                   "-c", src, "-o", obj]
            jobs.append(cmd)

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
        return res.stderr

    with concurrent.futures.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        for out in ex.map(run, jobs):
            if verbose and out:
                print(out)
    relink = jobs or not os.path.exists(LIB_PATH) or \
        os.path.getmtime(LIB_PATH) < max(os.path.getmtime(o) for o in objs)
    if relink:
        link = [nvcc, *ARCH_FLAGS, "-shared", "-o", LIB_PATH, *objs,
                "-Xlinker", f"-rpath={lib}", f"-L{lib}", "-l:libnccl.so.2",
                "-cudart", "static", "-lrt", "-ldl", "-lpthread"]
        run(link)
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
