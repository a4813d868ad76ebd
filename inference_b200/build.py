"""Build libq3_sm100a.so in-tree with nvcc for sm_100a.

    python -m inference_b200.build [--force] [-j N]

Each .cu (device + host) and .cpp (host only: the tokenizer) under csrc/
compiles to an object under inference_b200/_build/, then all link into
inference_b200/libq3_sm100a.so against the CUDA runtime (NCCL is
loaded at run time, only for tensor parallelism).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libq3_sm100a.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler",
                     "-fPIC,-fvisibility=hidden", "-I", os.path.join(ROOT, "include")]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found")
    return path


def _deps() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.hpp")) +
                  glob.glob(os.path.join(CSRC, "*.inc")) + glob.glob(os.path.join(ROOT, "include", "*.h")))


def _stale(out: str, srcs: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in srcs)


def build(force: bool = False, jobs: int = 8, verbose: bool = True, extra: list[str] | None = None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    deps = _deps()
    objs = []
    todo = []
    for src in sources:
        obj = os.path.join(BUILD, os.path.splitext(os.path.basename(src))[0] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src] + deps):
            todo.append((src, obj))

    def compile_one(item):
        src, obj = item
        cmd = [nvcc()] + NVCC_FLAGS + (extra or []) + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        return src, cmd, r

    failed = []
    with cf.ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        for src, cmd, r in ex.map(compile_one, todo):
            if verbose:
                print("nvcc", os.path.relpath(src, ROOT), flush=True)
            if r.returncode != 0:
                failed.append((src, r.stdout + r.stderr))
            elif verbose and r.stderr.strip():
                print(r.stderr, file=sys.stderr)
    if failed:
        for src, log in failed:
            print(f"--- {src}\n{log}", file=sys.stderr)
        raise RuntimeError(f"{len(failed)} CUDA source(s) failed to compile")
    if force or todo or _stale(LIB, objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart", "-ldl"]
        if verbose:
            print("link", os.path.relpath(LIB, ROOT), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=os.cpu_count() or 4)
    ap.add_argument("--ptxas-verbose", action="store_true")
    a = ap.parse_args(argv)
    build(a.force, a.jobs, extra=["-Xptxas", "-v"] if a.ptxas_verbose else None)
    return 0


if __name__ == "__main__":
    sys.exit(main())
