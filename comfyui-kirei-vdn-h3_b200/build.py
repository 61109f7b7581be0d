"""Build the in-tree sm_100a library ``libvdn_b200.so`` with nvcc.

    python comfyui-kirei-vdn-h3_b200/build.py [--force]

Every ``csrc/*.cu`` file is compiled for ``-gencode arch=compute_100a,code=sm_100a`` with
line info, then linked into one shared library next to this file (static cudart, so the
library does not depend on which libcudart the host process loaded).  Objects go to
``_build/`` and are rebuilt only when a source or header is newer.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libvdn_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the sm_100a library cannot be built")


def _newest_header() -> float:
    heads = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    return max((os.path.getmtime(h) for h in heads), default=0.0)


def _compile(src: str, obj: str, extra: list[str]) -> str:
    cmd = [_nvcc(), *ARCH, *FLAGS, *extra, "-c", src, "-o", obj]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{res.stderr}")
    return obj


def build(force: bool = False, extra_flags: list[str] | None = None, verbose: bool = False) -> str:
    """Compile and link the library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    extra = list(extra_flags or [])
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr = _newest_header()
    jobs = []
    objs = []
    for src in srcs:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        stale = force or not os.path.exists(obj) or os.path.getmtime(obj) < max(os.path.getmtime(src), hdr)
        if stale:
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for obj in ex.map(lambda j: _compile(j[0], j[1], extra), jobs):
                if verbose:
                    print("compiled", os.path.basename(obj))
    lib_stale = force or bool(jobs) or not os.path.exists(LIB) or any(
        os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs)
    if lib_stale:
        tmp = LIB + ".tmp"
        cmd = [_nvcc(), *ARCH, "-shared", "-o", tmp, *objs]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc link failed:\n{res.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    path = build(force=args.force, verbose=True)
    print(path)
    sys.exit(0)
