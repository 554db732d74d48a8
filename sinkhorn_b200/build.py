"""Build libsinkhorn_b200.so in-tree with nvcc for sm_100a.

    python -m sinkhorn_b200.build [--force] [--verbose]

Objects go to sinkhorn_b200/_build/, the library to
sinkhorn_b200/_lib/libsinkhorn_b200.so. Rebuilds only what changed (sources
or any header under csrc/ or include/).
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OBJ = os.path.join(PKG, "_build")
LIBDIR = os.path.join(PKG, "_lib")
LIBNAME = "libsinkhorn_b200.so"
LIB = os.path.join(LIBDIR, LIBNAME)

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3,-Wall", "-I" + os.path.join(ROOT, "include"),
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found (CUDA toolkit required to build sinkhorn_b200)")
    return cand


def _sources() -> list[str]:
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC)
                  if f.endswith((".cu", ".cpp")))


def _headers_mtime() -> float:
    t = 0.0
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh", ".hpp")):
                t = max(t, os.path.getmtime(os.path.join(d, f)))
    return t


def _compile(src: str, obj: str, ptxas_verbose: bool) -> tuple[str, str]:
    cmd = [nvcc()] + NVCC_FLAGS + ["-c", src, "-o", obj]
    if ptxas_verbose and src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}{r.stderr}")
    return src, r.stdout + r.stderr


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    hdr = _headers_mtime()
    jobs = []
    objs = []
    for src in _sources():
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        objs.append(obj)
        stale = (force or not os.path.exists(obj)
                 or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr))
        if stale:
            jobs.append((src, obj))
    with cf.ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        for src, log in ex.map(lambda j: _compile(j[0], j[1], ptxas_verbose), jobs):
            if verbose or ptxas_verbose:
                print(f"[nvcc] {os.path.basename(src)}\n{log}", end="")
    newest = max(os.path.getmtime(o) for o in objs)
    if force or jobs or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        tmp = LIB + ".tmp"
        cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
        os.replace(tmp, LIB)
        if verbose:
            print(f"[link] {LIB}")
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print -Xptxas -v register/smem usage")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, ptxas_verbose=a.ptxas))
    return 0


if __name__ == "__main__":
    sys.exit(main())
