"""Build libds_b200.so (all CUDA sources, sm_100a) into ds_b200/ in-tree.

    python ds-experiment_b200/build.py [--force] [-j N]

Every .cu under csrc/ is compiled with nvcc for sm_100a only
(-gencode arch=compute_100a,code=sm_100a), --fmad=false (no multiply is
contracted into an add unless the source asks for an FMA) and without
fast-math (IEEE division, no flush-to-zero), then linked into one shared
library with the static CUDA runtime.  Objects go to _build/ (git-ignored);
the .so lands next to the Python package so it travels with the tree.
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
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "ds_b200", "libds_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--fmad=false", "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden", "-I", INCLUDE, "-I", CSRC, "-I", BUILD,
    "-Xptxas", "-warn-spills", "--expt-relaxed-constexpr",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _compile(src, obj, extra):
    cmd = [nvcc()] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def _gen_arith_source():
    """ds_arith.cuh as a C++ raw string literal (the DS primitives that
    fuse.cu hands to NVRTC), without its include guard and CUDA header."""
    src = open(os.path.join(CSRC, "ds_arith.cuh")).read()
    body = "\n".join(l for l in src.splitlines()
                     if not l.startswith("#pragma once") and not l.startswith("#include"))
    text = 'R"DSARITH(' + body + '\n)DSARITH"\n'
    out = os.path.join(BUILD, "ds_arith_src.inc")
    if not os.path.exists(out) or open(out).read() != text:
        with open(out, "w") as f:
            f.write(text)


def build(force: bool = False, jobs: int = 0, verbose: bool = False, extra=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    _gen_arith_source()
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = _deps()
    objs = []
    todo = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.basename(src) + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + deps):
            todo.append((src, obj))
    if todo:
        jobs = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(jobs) as ex:
            for (src, _), log in zip(todo, ex.map(lambda t: _compile(t[0], t[1], list(extra)), todo)):
                if verbose and log.strip():
                    print(f"[{os.path.basename(src)}]\n{log}", file=sys.stderr)
    if force or todo or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lrt", "-lpthread", "-ldl"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=0)
    ap.add_argument("-v", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.j, verbose=args.v))
