"""Full-depth, long-context parity of the decode engine against the reference's
own CUDA backend (oracle/_ref/libref_cuda.so: cuBLAS GEMV + the reference's
kernels, built from its sources for sm_100a), with the reference's own
CUDA-vs-CPU spread measured in the same run.  TEST INFRASTRUCTURE (run by
tests/test_gpu_parity_full.py, one case per process).

One case = one configuration of the decode benchmark at its real depth and
context:

* The reference CUDA model consumes the prompt one Model::forward at a time
  (Model::prefill, src/lib/model/qwen3/qwen3.hpp:168-173) and then decodes
  greedily to the context limit (the Generator loop,
  src/lib/inference/generator.cpp:47-56, EOS ignored).  Its ids define the
  teacher-forced sequence S.
* The engine runs its own path on S in lockstep: batched prefill of the
  prompt, then one decode step per position consuming S (teacher forcing), so
  every decode step's logits are compared with the reference's, on
  independently computed KV histories.
* The reference's CPU backend (libref_cpu.so) measures the reference's own
  implementation spread: on its own history (like the engine) from the start
  for as many decode steps as the CPU can afford (the whole window for
  Qwen3-0.6B to context 1024), then over windows of WINDOW steps that start
  from the reference CUDA model's KV cache copied in (shared history).  A
  second engine starts each window from the same copied cache, so its spread
  is measured exactly like the CPU's.

The reference CUDA backend sizes its attention scratch once per process, from
its first call's query heads and cache length
(src/lib/backend/cuda/backend.cu:87-91,122-133): one model per process.

    python tests/parity_full.py CASE [--json OUT]
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

# name -> (model, prompt tokens, context, decode steps the reference CPU model runs on its own
# history from the start (all of them for the smallest model), shared-history window starts)
CASES = {
    "qwen3-0.6b-ctx1024": ("qwen3-0.6b", 16, 1024, 1008, []),
    "qwen3-0.6b-ctx8192": ("qwen3-0.6b", 4096, 8192, 0, [4095, 8158]),
    "qwen3-4b-ctx4096": ("qwen3-4b", 128, 4096, 160, [2100, 4062]),
    "qwen3-8b-ctx4096": ("qwen3-8b", 512, 4096, 128, [2300, 4062]),
}
WINDOW = 32


def bf(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def bf16_ulp(x: np.ndarray) -> np.ndarray:
    x = np.maximum(np.abs(np.asarray(x, np.float64)), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(x)) - 7)


class Pair:
    """Per-step logit agreement of one implementation with the reference CUDA model."""

    def __init__(self):
        self.rows = []  # per step: [position, max|d|, mean|d|, max(|d| - ulp(ref)), cosine, ref top-2 margin, agree]

    def add(self, mine_bits, ref_bits, next_token, step):
        m, r = bf(mine_bits).astype(np.float64), bf(ref_bits).astype(np.float64)
        d = np.abs(m - r)
        cos = float(m @ r / (np.linalg.norm(m) * np.linalg.norm(r) + 1e-30))
        top2 = np.partition(r, -2)[-2:]
        agree = int(int(np.argmax(m)) == int(next_token))  # first index of the maximum
        self.rows.append([step, float(d.max()), float(d.mean()), float((d - bf16_ulp(r)).max()), cos,
                          float(top2[1] - top2[0]), agree])

    def summary(self):
        if not self.rows:
            return None
        a = np.array(self.rows)
        return {"steps": len(a), "maxabs": round(float(a[:, 1].max()), 6), "meanabs": float(a[:, 2].mean()),
                "excess_over_ulp": round(float(a[:, 3].max()), 6), "mincos": round(float(a[:, 4].min()), 8),
                "agree": int(a[:, 6].sum()), "worst_step": int(a[int(a[:, 1].argmax()), 0])}

    def table(self):
        """The per-step rows, compact, for the test's paired statistics."""
        return [[int(r[0]), round(r[1], 6), round(r[2], 8), round(r[3], 6), round(r[4], 9), round(r[5], 6),
                 int(r[6])] for r in self.rows]


def run(case: str) -> dict:
    from inference_b200 import MODELS, Engine, prompt_ids
    from oracle import ModelConfig, RefLib

    model, P, C, cpu_indep, windows = CASES[case]
    cfg = MODELS[model]
    t_start = time.time()
    mc = ModelConfig.make(cfg.hidden, cfg.inter, cfg.layers, cfg.q_heads, cfg.kv_heads, 128, cfg.vocab, C,
                          tied=cfg.tied)
    ref = RefLib("cuda").model(mc, seed=0)
    cpu = RefLib("cpu").model(mc, seed=0)
    prompt = prompt_ids(P, seed=1, vocab=cfg.vocab).astype(np.uint32)
    S = np.zeros(C, np.uint32)
    S[:P] = prompt

    eng = Engine(cfg, capacity=C)
    eng.init_synthetic(0)
    eng.set_tokens(prompt)
    eng.prefill(P - 1)
    eng2 = None
    if windows:
        eng2 = Engine(cfg, capacity=C)
        eng2.init_synthetic(0)

    # the reference prefills one forward per prompt token (the CPU model too when it starts
    # on its own history)
    for p in range(P - 1):
        ref.forward(int(S[p]))
        if cpu_indep:
            cpu.forward(int(S[p]))
    t_pre = time.time()

    engine_pair, cpu_indep_pair, cpu_shared_pair, eng2_pair = Pair(), Pair(), Pair(), Pair()
    win_pairs = {}
    active = None  # (start, cpu, engine 2, engine) Pairs of the running window
    for p in range(P - 1, C - 1):
        if active is None and p in windows:
            # shared history: the reference CUDA model's KV cache [0, p) into the CPU model and engine 2
            for layer in range(cfg.layers):
                k, v = ref.kv_read(layer, 0, p)
                cpu.kv_write(layer, 0, k, v)
                eng2.kv_write(layer, 0, k, v)
            cpu.token_count = p
            eng2.set_position(p)
            active = (p, Pair(), Pair(), Pair())
            win_pairs[p] = active
        nxt = ref.forward(int(S[p]))
        S[p + 1] = nxt
        r_logits = ref.logits()
        eng.set_tokens(S[: p + 1])
        eng.step(1)
        eng.sync()
        e1 = eng.logits()
        engine_pair.add(e1, r_logits, nxt, p)
        if p < P - 1 + cpu_indep:
            cpu.forward(int(S[p]))
            cpu_indep_pair.add(cpu.logits(), r_logits, nxt, p)
        if active:
            cpu.forward(int(S[p]))
            c_logits = cpu.logits()
            cpu_shared_pair.add(c_logits, r_logits, nxt, p)
            active[1].add(c_logits, r_logits, nxt, p)
            active[3].add(e1, r_logits, nxt, p)
            eng2.set_tokens(S[: p + 1])
            eng2.step(1)
            eng2.sync()
            e2 = eng2.logits()
            eng2_pair.add(e2, r_logits, nxt, p)
            active[2].add(e2, r_logits, nxt, p)
            if p + 1 - active[0] >= WINDOW:
                active = None
    # the engine's fused greedy argmax by position (bit-exact against the argmax of its logits)
    hist = eng.argmax_history(C - 1)
    ref.close()
    cpu.close()
    eng.close()
    if eng2:
        eng2.close()
    return {
        "case": case, "model": model, "layers": cfg.layers, "prompt": P, "context": C, "decode_steps": C - P,
        "cpu": f"own history for the first {cpu_indep} decode steps; shared-history windows of {WINDOW} at "
               f"{windows}",
        "engine_vs_ref_cuda": engine_pair.summary(),
        "ref_cpu_vs_ref_cuda_own_history": cpu_indep_pair.summary(),
        "ref_cpu_vs_ref_cuda_shared_history": cpu_shared_pair.summary(),
        "engine_shared_history_vs_ref_cuda": eng2_pair.summary(),
        "windows": {str(k): {"ref_cpu": v[1].summary(), "engine_shared": v[2].summary(),
                             "engine": v[3].summary()}
                    for k, v in win_pairs.items()},
        "rows": {"engine": engine_pair.table(), "ref_cpu_own": cpu_indep_pair.table(),
                 "ref_cpu_shared": cpu_shared_pair.table(), "engine_shared": eng2_pair.table()},
        "row_fields": ["position", "maxabs", "meanabs", "excess_over_ulp", "cosine", "ref_top2_margin", "agree"],
        "sequence_head": [int(x) for x in S[P:P + 8]],
        "engine_greedy_vs_sequence": int((hist[P - 1:C - 1] == S[P:C]).sum()),
        "seconds": {"prefill": round(t_pre - t_start, 1), "total": round(time.time() - t_start, 1)},
    }


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=sorted(CASES))
    ap.add_argument("--json", default=None)
    a = ap.parse_args(argv)
    out = run(a.case)
    line = json.dumps(out)
    print(line, flush=True)
    if a.json:
        with open(a.json, "w") as f:
            f.write(line + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
