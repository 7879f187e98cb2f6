"""Builds the native library `objectsam_b200/libosam.so` from `objectsam_b200/csrc` with nvcc for sm_100a.

Each translation unit is compiled to an object file under `objectsam_b200/_build/` (rebuilt only when the
source or any header in csrc/ or include/ is newer), then linked into one shared library with a static
CUDA runtime.  Run `python -m objectsam_b200.build` or call `build()`.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD_DIR = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libosam.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
    "--expt-relaxed-constexpr", "-I" + INCLUDE, "-I" + CSRC,
]

# Files compiled under extra flags.  augment.cu restates the reference's augmentation float steps, which
# the reference compiles with --use_fast_math (its Release flags): the same flags make the same roundings
# (division, flush-to-zero), so pixels, boxes and mask bits agree bit for bit.
FILE_FLAGS = {"augment.cu": ["--use_fast_math"]}


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    out = []
    for dirpath, _, files in os.walk(CSRC):
        for f in sorted(files):
            if f.endswith((".cu", ".cpp")):
                out.append(os.path.join(dirpath, f))
    return sorted(out)


def _headers():
    hs = []
    for d in (CSRC, INCLUDE):
        for dirpath, _, files in os.walk(d):
            hs += [os.path.join(dirpath, f) for f in files if f.endswith((".h", ".cuh", ".hpp"))]
    return hs


def _compile(src: str, newest_header: float, verbose: bool) -> str:
    rel = os.path.relpath(src, CSRC).replace(os.sep, "_")
    obj = os.path.join(BUILD_DIR, rel + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), newest_header):
        return obj
    cmd = [nvcc()] + NVCC_FLAGS + FILE_FLAGS.get(os.path.basename(src), []) + ["-x", "cu", "-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr.strip():
        print(res.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False, jobs: int | None = None) -> str:
    """Compile every CUDA/C++ source of the package for sm_100a and link libosam.so; returns its path."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    srcs = _sources()
    newest_header = max([os.path.getmtime(h) for h in _headers()] + [0.0])
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, newest_header, verbose), srcs))
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "static", "-o", LIB] + objs
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
