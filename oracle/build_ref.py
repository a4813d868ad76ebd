"""Build recipe for the oracle libraries.  TEST INFRASTRUCTURE ONLY.

* ``oracle/libq3_oracle.so`` -- the C restatement (q3_oracle.c).  Needs only gcc.
* ``oracle/_ref/libref_cpu.so`` -- the reference's own AVX-512 CPU backend and
  Qwen3 model, compiled from the reference sources where they lie (never
  copied), with the flags of src/lib/backend/cpu/CMakeLists.txt:7-15, plus
  ref_harness.cpp as a C-ABI driver.  Built only where the reference tree is
  present; the output travels with the repository snapshot.
* ``oracle/_ref/libref_cuda.so`` -- the reference's cuBLAS CUDA backend built
  the same way for sm_100a.  It needs CCCL >= 3 headers (cuda::launch,
  cuda::device_memory_pool); CUDA 12.9 ships CCCL 2.8, so the CCCL 3.x tree
  bundled with flashinfer is used when present.
* ``oracle/_ref/libref_b200.so`` -- the same harness and the reference's own
  Qwen3 model, with this repository's drop-in Backend
  (inference_b200/backend_b200/backend.cpp) linked in place of the reference's
  CUDA backend: the reference's Model::forward running on libq3_sm100a.so.

Run: ``python oracle/build_ref.py [--reference DIR] [--no-cuda]``.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REF_OUT = os.path.join(HERE, "_ref")
DEFAULT_REFERENCE = "/root/reference"


def reference_dir() -> str:
    """Where the reference's sources are read from: $Q3_REFERENCE_DIR if set,
    else this recipe's default location."""
    return os.environ.get("Q3_REFERENCE_DIR") or DEFAULT_REFERENCE


def _site_packages() -> str:
    import sysconfig

    return sysconfig.get_paths()["purelib"]


def _nlohmann_include() -> str | None:
    cand = os.path.join(_site_packages(), "include", "cudnn_frontend", "thirdparty")
    return cand if os.path.isfile(os.path.join(cand, "nlohmann", "json.hpp")) else None


def _cccl3_includes() -> list[str] | None:
    root = os.path.join(_site_packages(), "flashinfer", "data", "cccl")
    parts = [os.path.join(root, "libcudacxx", "include"), os.path.join(root, "cub"), os.path.join(root, "thrust")]
    if all(os.path.isdir(p) for p in parts) and os.path.isfile(os.path.join(parts[0], "cuda", "launch")):
        return parts
    return None


def _run(cmd: list[str]) -> None:
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)


def _newer(out: str, srcs: list[str]) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(s) <= t for s in srcs if os.path.exists(s))


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "q3_oracle.c")
    out = os.path.join(HERE, "libq3_oracle.so")
    if force or not _newer(out, [src]):
        _run(["gcc", "-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC",
              "-shared", "-fvisibility=hidden", "-std=c11", src, "-o", out, "-lm"])
    return out


def build_ref_cpu(reference: str, force: bool = False) -> str | None:
    lib = os.path.join(reference, "src", "lib")
    backend_cpp = os.path.join(lib, "backend", "cpu", "backend.cpp")
    nl = _nlohmann_include()
    if not os.path.isfile(backend_cpp) or nl is None:
        print("reference CPU backend not buildable here (sources or nlohmann/json missing)")
        return None
    os.makedirs(REF_OUT, exist_ok=True)
    out = os.path.join(REF_OUT, "libref_cpu.so")
    harness = os.path.join(HERE, "ref_harness.cpp")
    compat = os.path.join(HERE, "ref_compat.hpp")
    if force or not _newer(out, [harness, compat, backend_cpp]):
        # Flags from src/lib/backend/cpu/CMakeLists.txt:1-17 (-march=x86-64-v4
        # -mavx512bf16 -ffast-math + OpenMP) and CMakeLists.txt (C++23).
        _run(["g++", "-std=c++23", "-O3", "-march=x86-64-v4", "-mavx512bf16", "-ffast-math", "-fopenmp", "-fPIC",
              "-shared", "-include", compat, "-I", lib, "-I", nl, harness, backend_cpp,
              "-L", HERE, "-lq3_oracle", "-Wl,-rpath,$ORIGIN/..", "-o", out])
    return out


def build_ref_cuda(reference: str, force: bool = False) -> str | None:
    lib = os.path.join(reference, "src", "lib")
    backend_cu = os.path.join(lib, "backend", "cuda", "backend.cu")
    nl = _nlohmann_include()
    cccl = _cccl3_includes()
    if not os.path.isfile(backend_cu) or nl is None or cccl is None or shutil.which("nvcc") is None:
        print("reference CUDA backend not buildable here (sources, nlohmann/json, CCCL 3.x or nvcc missing)")
        return None
    os.makedirs(REF_OUT, exist_ok=True)
    out = os.path.join(REF_OUT, "libref_cuda.so")
    harness = os.path.join(HERE, "ref_harness.cpp")
    if force or not _newer(out, [harness, backend_cu]):
        obj_dir = os.path.join(REF_OUT, "obj")
        os.makedirs(obj_dir, exist_ok=True)
        inc = []
        for p in cccl:
            inc += ["-I", p]
        common = ["-std=c++20", "-O3", "-gencode", "arch=compute_100a,code=sm_100a", "--expt-relaxed-constexpr",
                  "--extended-lambda", "-Xcompiler", "-fPIC", "-I", lib, "-I", nl] + inc
        o1 = os.path.join(obj_dir, "backend_cuda.o")
        o2 = os.path.join(obj_dir, "harness_cuda.o")
        # backend.cu is the reference's only CUDA translation unit (C++20,
        # src/lib/backend/cuda/CMakeLists.txt:18-22); the model code is host
        # C++23 (std::views::zip), compiled by g++ as the reference's CMake does.
        _run(["nvcc"] + common + ["-c", backend_cu, "-o", o1])
        cuda_inc = os.path.join(os.path.dirname(os.path.dirname(shutil.which("nvcc"))), "include")
        _run(["g++", "-std=c++23", "-O2", "-fPIC", "-DREF_CUDA", "-I", lib, "-I", nl, "-I", cuda_inc, "-c", harness,
              "-o", o2])
        cuda_lib = os.path.join(os.path.dirname(cuda_inc), "lib64")
        _run(["g++", "-shared", o1, o2, "-o", out, "-L", HERE, "-lq3_oracle", "-Wl,-rpath,$ORIGIN/..",
              "-L", cuda_lib, "-lcublas", "-lcudart"])
    return out


def build_ref_b200(reference: str, force: bool = False) -> str | None:
    lib = os.path.join(reference, "src", "lib")
    repo = os.path.dirname(HERE)
    backend_cpp = os.path.join(repo, "inference_b200", "backend_b200", "backend.cpp")
    q3_lib = os.path.join(repo, "inference_b200", "libq3_sm100a.so")
    nl = _nlohmann_include()
    nvcc = shutil.which("nvcc")
    if not os.path.isdir(lib) or nl is None or nvcc is None or not os.path.isfile(q3_lib):
        print("drop-in backend harness not buildable here (reference tree, nlohmann/json, nvcc or "
              "libq3_sm100a.so missing)")
        return None
    os.makedirs(REF_OUT, exist_ok=True)
    out = os.path.join(REF_OUT, "libref_b200.so")
    harness = os.path.join(HERE, "ref_harness.cpp")
    header = os.path.join(repo, "include", "q3_sm100a.h")
    if force or not _newer(out, [harness, backend_cpp, header, q3_lib]):
        obj_dir = os.path.join(REF_OUT, "obj")
        os.makedirs(obj_dir, exist_ok=True)
        cuda_inc = os.path.join(os.path.dirname(os.path.dirname(nvcc)), "include")
        cuda_lib = os.path.join(os.path.dirname(cuda_inc), "lib64")
        flags = ["g++", "-std=c++23", "-O2", "-fPIC", "-I", lib, "-I", nl, "-I", cuda_inc]
        o1 = os.path.join(obj_dir, "backend_b200.o")
        o2 = os.path.join(obj_dir, "harness_b200.o")
        _run(flags + ["-I", os.path.join(repo, "include"), "-c", backend_cpp, "-o", o1])
        _run(flags + ["-DREF_CUDA", "-c", harness, "-o", o2])
        _run(["g++", "-shared", o1, o2, "-o", out, "-L", HERE, "-lq3_oracle",
              "-L", os.path.dirname(q3_lib), "-lq3_sm100a",
              "-Wl,-rpath,$ORIGIN/..:$ORIGIN/../../inference_b200", "-L", cuda_lib, "-lcudart"])
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None, help="reference source tree (default: $Q3_REFERENCE_DIR, "
                    "else the recipe's default location)")
    ap.add_argument("--no-cuda", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args(argv)
    a.reference = a.reference or reference_dir()
    build_oracle(a.force)
    if os.path.isdir(a.reference):
        build_ref_cpu(a.reference, a.force)
        if not a.no_cuda:
            try:
                build_ref_cuda(a.reference, a.force)
            except subprocess.CalledProcessError as e:  # optional GPU oracle
                print("reference CUDA backend build failed:", e)
            try:
                build_ref_b200(a.reference, a.force)
            except subprocess.CalledProcessError as e:
                print("drop-in backend harness build failed:", e)
    else:
        print("reference tree absent: using prebuilt oracle/_ref libraries if any")
    return 0


if __name__ == "__main__":
    sys.exit(main())
