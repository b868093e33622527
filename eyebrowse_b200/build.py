"""Build libeyebrowse_attn.so (the C-ABI library) in-tree for sm_100a.

    python -m eyebrowse_b200.build        # or: from eyebrowse_b200.build import build

Each .cu under csrc/ compiles to an object in parallel; the objects link into
eyebrowse_b200/libeyebrowse_attn.so with the CUDA runtime linked statically,
so the library loads in any process (with or without torch) on the GPU box.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libeyebrowse_attn.so")
ROOT = os.path.dirname(HERE)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
                     "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def nvcc() -> str:
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(p):
        raise RuntimeError("nvcc not found")
    return p


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hs.append(os.path.join(ROOT, "include", "eyebrowse_attn.h"))
    return hs


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool, extra) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    if _stale(obj, [src] + _headers()):
        cmd = [nvcc()] + NVCC_FLAGS + list(extra) + ["-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and r.stderr.strip():
            print(r.stderr, flush=True)
    return obj


def build(verbose: bool = False, extra=()) -> str:
    """Compile every CUDA source for sm_100a and link the shared library."""
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, extra), srcs))
    if _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + ["-cudart", "static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    return LIB


def build_shared(src: str, out: str, verbose: bool = False) -> str:
    """Compile one standalone .cu (e.g. a test-only diagnostic) into a shared library."""
    if _stale(out, [src] + _headers()):
        cmd = [nvcc()] + NVCC_FLAGS + ["-shared", "-o", out, src, "-cudart", "static"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return out


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, extra=["-Xptxas", "-v"] if "--ptxas" in sys.argv else ())
    print(LIB)
