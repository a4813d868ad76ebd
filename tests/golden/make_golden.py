"""Generate the golden fixtures from the REFERENCE's own CPU backend.

Runs the reference's AVX-512 CPU backend and Qwen3 model (compiled from its
sources by oracle/build_ref.py into oracle/_ref/libref_cpu.so) on seeded
inputs and stores its outputs under tests/golden/.  Inputs are regenerated
from seeds by tests/golden/inputs.py (kernel cases) or by the synthetic
weight generator (model cases), so the fixtures hold outputs only.

Run here, where the reference tree exists:
    python oracle/build_ref.py && python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

from inputs import uniform_bf16  # noqa: E402
from oracle import ModelConfig, Oracle, RefLib  # noqa: E402

# Kernel cases: the reference's own test shapes (testing/tests/*.cpp, listed
# beside each) plus the Qwen3 shapes the decode path runs at.
GEMV = [(i, o) for i in (32, 64, 128) for o in (1, 7, 8, 9)] + [(1024, 2048), (2560, 1024), (4096, 1024),
                                                                 (3072, 1024), (1024, 4096)]  # gemv.cpp:25-26
NORM = [128, 256, 1024, 2560, 4096, 5120]  # rmsnorm.cpp:25
QKNR = [(8, 2, 0), (8, 2, 1), (8, 2, 50), (8, 8, 0), (8, 8, 1), (8, 8, 50),  # qk_norm_rope.cpp:27-29
        (16, 8, 1000), (32, 8, 4095), (64, 8, 8191)]
ATTN = [(32, 32, 1024),  # self_attention.cpp:18-21 (no GQA)
        (16, 8, 0), (16, 8, 1023), (32, 8, 300), (64, 8, 77), (32, 8, 4095), (16, 8, 8191)]
ELEM = [1, 15, 16, 17, 255, 256, 257, 3072]  # add.cpp:22
ARGMAX = [1, 15, 16, 17, 255, 256, 257, 151936]  # sampling.cpp:19

MODELS = {
    # name: (config, prompt_len, decode_steps)
    "qwen3_0p6b": (ModelConfig.make(1024, 3072, 28, 16, 8, 128, 151936, 64, tied=True), 16, 8),
    "qwen3_4b_l2": (ModelConfig.make(2560, 9728, 2, 32, 8, 128, 151936, 32, tied=True), 8, 4),
    "qwen3_8b_l2": (ModelConfig.make(4096, 12288, 2, 32, 8, 128, 151936, 32, tied=False), 8, 4),
    "qwen3_32b_l1": (ModelConfig.make(5120, 25600, 1, 64, 8, 128, 151936, 16, tied=False), 4, 2),
}
TOPK = 16


def seed_of(*parts) -> int:
    h = 1469598103934665603
    for p in parts:
        for ch in str(p).encode():
            h = ((h ^ ch) * 1099511628211) & 0xFFFFFFFFFFFF
    return h


def kernel_cases(ref: RefLib) -> dict:
    out = {}
    for i, o in GEMV:
        x = uniform_bf16(seed_of("gemv.x", i, o), (i,))
        w = uniform_bf16(seed_of("gemv.w", i, o), (o, i))
        out[f"gemv/{i}x{o}"] = ref.gemv(x, w)
    for h in NORM:
        x = uniform_bf16(seed_of("norm.x", h), (h,))
        w = uniform_bf16(seed_of("norm.w", h), (h,))
        u = uniform_bf16(seed_of("norm.u", h), (h,))
        out[f"rmsnorm/{h}"] = ref.rmsnorm(x, w)
        res, o2 = ref.rmsnorm_add(x, u, w)
        out[f"rmsnorm_add_res/{h}"] = res
        out[f"rmsnorm_add_out/{h}"] = o2
    for qh, kvh, pos in QKNR:
        q = uniform_bf16(seed_of("qknr.q", qh, kvh, pos), (qh, 128))
        k = uniform_bf16(seed_of("qknr.k", qh, kvh, pos), (kvh, 128))
        qn = uniform_bf16(seed_of("qknr.qn", qh, kvh, pos), (128,))
        kn = uniform_bf16(seed_of("qknr.kn", qh, kvh, pos), (128,))
        q2, k2 = ref.qk_norm_rope(q, k, qn, kn, pos)
        out[f"qknr_q/{qh}_{kvh}_{pos}"] = q2
        out[f"qknr_k/{qh}_{kvh}_{pos}"] = k2
    for qh, kvh, pos in ATTN:
        q = uniform_bf16(seed_of("attn.q", qh, kvh, pos), (qh, 128))
        kc = uniform_bf16(seed_of("attn.k", qh, kvh, pos), (pos + 1, kvh, 128))
        vc = uniform_bf16(seed_of("attn.v", qh, kvh, pos), (pos + 1, kvh, 128))
        out[f"attn/{qh}_{kvh}_{pos}"] = ref.attention(q, kc, vc, pos)
    for n in ELEM:
        a = uniform_bf16(seed_of("elem.a", n), (n,))
        b = uniform_bf16(seed_of("elem.b", n), (n,))
        out[f"silu/{n}"] = ref.silu(a, b)
        out[f"add/{n}"] = ref.add(a, b)
    for n in ARGMAX:
        lg = uniform_bf16(seed_of("argmax", n), (n,))
        out[f"argmax/{n}"] = np.array([ref.argmax(lg)], np.int64)
    # ties: the maximum appears several times; the first index must win.
    lg = uniform_bf16(seed_of("argmax.tie"), (4099,), -2.0, 1.0)
    lg[[17, 1000, 4098]] = 0x4040  # 3.0
    out["argmax_tie/4099"] = np.array([ref.argmax(lg)], np.int64)
    table = uniform_bf16(seed_of("embed"), (64, 1024))
    out["embedding/37"] = ref.embedding(37, table)
    c, s = ref.rope_cache(4096)
    rows = np.array([0, 1, 2, 511, 1023, 2047, 4095])
    out["rope_cos_rows"] = c[rows]
    out["rope_sin_rows"] = s[rows]
    return out


def model_case(ref: RefLib, o: Oracle, name: str) -> dict:
    cfg, plen, steps = MODELS[name]
    prompt = o.prompt_ids(plen, seed=1, vocab=cfg.vocab)
    t0 = time.time()
    m = ref.model(cfg, seed=0)
    om = o.model(cfg, seed=0)  # the oracle in lockstep: the envelope two fp32 implementations span
    env_max, env_cos = [], []
    seq = list(int(t) for t in prompt)
    argmax, topi, topv, s1, s2 = [], [], [], [], []
    kv_layers = sorted({0, cfg.layers - 1})
    kv = {lay: ([], []) for lay in kv_layers}
    n_fwd = plen + steps
    for i in range(n_fwd):
        nxt = m.forward(seq[i])
        lg = m.logits()
        f = (lg.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        om.forward(seq[i])
        fo = (om.logits().astype(np.uint32) << 16).view(np.float32).astype(np.float64)
        env_max.append(float(np.abs(f - fo).max()))
        env_cos.append(float(f @ fo / (np.linalg.norm(f) * np.linalg.norm(fo))))
        idx = np.argsort(-f, kind="stable")[:TOPK]
        argmax.append(nxt)
        topi.append(idx.astype(np.int64))
        topv.append(lg[idx])
        s1.append(f.sum())
        s2.append((f * f).sum())
        for lay in kv_layers:
            k, v = m.kv_slot(lay, i)
            kv[lay][0].append(k)
            kv[lay][1].append(v)
        if i >= plen - 1 and len(seq) < n_fwd:
            seq.append(nxt)
    m.close()
    om.close()
    print(f"  {name}: {n_fwd} forwards in {time.time() - t0:.1f}s; reference CPU vs oracle: max |dlogit| "
          f"{max(env_max):.4f}, min cosine {min(env_cos):.6f}", flush=True)
    d = {
        "config": np.array([cfg.hidden, cfg.inter, cfg.layers, cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.vocab,
                            cfg.capacity, cfg.tied], np.int64),
        "tokens": np.array(seq, np.int64),
        "prompt_len": np.array([plen], np.int64),
        "argmax": np.array(argmax, np.int64),
        "top_idx": np.stack(topi),
        "top_val": np.stack(topv),
        "logit_sum": np.array(s1),
        "logit_sumsq": np.array(s2),
        "kv_layers": np.array(kv_layers, np.int64),
        # per step: max |logit difference| and cosine between the reference
        # CPU backend and the oracle -- how far apart two correct fp32
        # implementations of the same model land
        "env_maxabs": np.array(env_max),
        "env_cos": np.array(env_cos),
    }
    for lay in kv_layers:
        d[f"k_l{lay}"] = np.stack(kv[lay][0])
        d[f"v_l{lay}"] = np.stack(kv[lay][1])
    return d


def main():
    ref = RefLib("cpu")
    o = Oracle()
    print("kernel cases", flush=True)
    np.savez_compressed(os.path.join(HERE, "ops_ref_cpu.npz"), **kernel_cases(ref))
    for name in MODELS:
        print("model", name, flush=True)
        np.savez_compressed(os.path.join(HERE, f"model_{name}_ref_cpu.npz"), **model_case(ref, o, name))


if __name__ == "__main__":
    main()
