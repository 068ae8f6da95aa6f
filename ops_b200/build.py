"""Build libsfa_b200.so (the C-ABI library) in-tree for sm_100a with nvcc.

    python -m ops_b200.build [--force] [--jobs N]

Objects go to ops_b200/_build/, the shared library to ops_b200/libsfa_b200.so.
The library links only the CUDA runtime (static) — no torch, no Python.
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libsfa_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _flags():
    return ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr",
                   "-I" + os.path.join(ROOT, "include"), "-I" + CSRC, "-DNDEBUG"]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) +
                  glob.glob(os.path.join(ROOT, "include", "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, jobs: int = 0, verbose: bool = False, extra: list | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    nvcc = nvcc_path()
    headers = _headers()
    srcs = _sources()
    objs = []
    cmds = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmds.append([nvcc, "-c", s, "-o", o] + _flags() + list(extra or []))

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)
        if verbose and (r.stdout or r.stderr):
            sys.stderr.write(r.stdout + r.stderr)

    if cmds:
        with ThreadPoolExecutor(max_workers=jobs or min(len(cmds), os.cpu_count() or 4)) as ex:
            list(ex.map(run, cmds))
    if force or cmds or _stale(LIB, objs):
        run([nvcc, "-shared", "-o", LIB] + objs + ARCH + ["-Xcompiler", "-fPIC", "-cudart", "static"])
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=0)
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/spill info")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_info else None
    print(build(force=a.force or a.ptxas_info, jobs=a.jobs, verbose=a.verbose or a.ptxas_info, extra=extra))


if __name__ == "__main__":
    main()
