"""The reference's own CUDA backend on the golden model records (run on a B200).

For each model record tests/golden/model_<name>_ref_cpu.npz this teacher-forces
the reference's cuBLAS CUDA backend (oracle/_ref/libref_cuda.so, built from
the reference's sources) on the record's tokens and writes, per step, its
distance from the oracle model (max |logit difference|, cosine) and its greedy
token to tests/golden/model_<name>_ref_cuda.npz.  A GPU implementation's
distance from the oracle is the comparison for the engine's: the oracle
restates the reference CPU backend's arithmetic in its own lane order, so the
reference CPU backend sits closer to it than any GPU implementation does.

    python tests/golden/make_golden_cuda.py [NAME ...]

Each record runs in its own process: the reference CUDA backend sizes its
attention scratch once per process from its first call
(src/lib/backend/cuda/backend.cu:87-91,122-133).
"""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
NAMES = ["qwen3_0p6b", "qwen3_4b_l2", "qwen3_8b_l2", "qwen3_32b_l1"]


def bf(a):
    return (np.asarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32).astype(np.float64)


def one(name: str) -> None:
    sys.path.insert(0, ROOT)
    from oracle import ModelConfig, Oracle, RefLib

    g = dict(np.load(os.path.join(HERE, f"model_{name}_ref_cpu.npz")))
    h, inter, layers, qh, kvh, hd, vocab, cap, tied = (int(v) for v in g["config"])
    mc = ModelConfig.make(h, inter, layers, qh, kvh, hd, vocab, cap, tied=bool(tied))
    rm = RefLib("cuda").model(mc, seed=0)
    om = Oracle().model(mc, seed=0)
    maxabs, cos, argmax = [], [], []
    for t in g["tokens"]:
        argmax.append(rm.forward(int(t)))
        om.forward(int(t))
        r, o = bf(rm.logits()), bf(om.logits())
        maxabs.append(float(np.abs(r - o).max()))
        cos.append(float(r @ o / (np.linalg.norm(r) * np.linalg.norm(o))))
    rm.close()
    om.close()
    out = os.path.join(HERE, f"model_{name}_ref_cuda.npz")
    np.savez(out, cuda_maxabs=np.array(maxabs), cuda_cos=np.array(cos), cuda_argmax=np.array(argmax, np.int64))
    print(f"{name}: reference CUDA vs oracle max |d| {max(maxabs):.4f}, min cosine {min(cos):.6f} -> {out}")


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    if len(argv) == 2 and argv[0] == "--one":
        one(argv[1])
        return 0
    for name in argv or NAMES:
        subprocess.run([sys.executable, os.path.abspath(__file__), "--one", name], check=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
