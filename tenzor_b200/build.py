"""Builds libtenzor_cuda.so in-tree for sm_100a (nvcc cross-compiles; no GPU needed).

    python -m tenzor_b200.build [--force] [--verbose]

Each translation unit under csrc/ is compiled with
``nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` into csrc/_build/, then linked into
tenzor_b200/libtenzor_cuda.so (static cudart; the driver API is reached through
cudaGetDriverEntryPoint, so there is no libcuda link dependency).  Rebuilds only what changed.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(CSRC, "_build")
LIB = os.path.join(PKG, "libtenzor_cuda.so")
INCLUDE = os.path.join(os.path.dirname(PKG), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills", f"-I{INCLUDE}"]


def nvcc() -> str:
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(p):
        raise RuntimeError("nvcc not found")
    return p


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _headers_mtime():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs.append(os.path.join(INCLUDE, "tenzor_cuda.h"))
    return max(os.path.getmtime(h) for h in hs)


def _compile(src: str, force: bool, verbose: bool, extra):
    obj = os.path.join(BUILD, src + ".o")
    path = os.path.join(CSRC, src)
    if not force and os.path.exists(obj):
        if os.path.getmtime(obj) >= max(os.path.getmtime(path), _headers_mtime()):
            return obj, None
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", path, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [nvcc(), *NVCC_FLAGS, *extra, "-x", "c++", "-c", path, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    out = (r.stdout or "") + (r.stderr or "")
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{out}")
    return obj, out if verbose else None


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, force, verbose, list(extra)), srcs))
    objs = [o for o, _ in results]
    for o, log in results:
        if log:
            print(f"== {os.path.basename(o)}\n{log}")
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs, "-Xcompiler", "-fPIC"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/spill reports")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.verbose else []
    print(build(force=a.force or a.verbose, verbose=a.verbose, extra=extra))


if __name__ == "__main__":
    sys.exit(main())
