"""Batched prefill (tcgen05 GEMMs + batched attention) against the oracle and
against the engine's own per-token decode step.

The reference prefills with one decode forward per prompt token
(qwen3.hpp:168-173) and discards the logits, so the prefill's observable
result is the KV cache: it is compared slot by slot with the oracle and the
reference CPU fixture, and every logit of the decode steps that follow (which
attend over the prefilled cache) is held to the teacher-forced engine bound
(test_gpu_engine.py).
"""
import os

import numpy as np
import pytest

from gpu_util import assert_logits_close, assert_within_spread, bf, paired_no_worse, spread_of

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _cfgs(name):
    from inference_b200 import Qwen3Config
    from oracle import ModelConfig

    g = dict(np.load(os.path.join(GOLD, f"model_{name}_ref_cpu.npz")))
    h, inter, layers, qh, kvh, hd, vocab, cap, tied = (int(v) for v in g["config"])
    qc = Qwen3Config(name, hidden=h, inter=inter, layers=layers, q_heads=qh, kv_heads=kvh, vocab=vocab,
                     tied=bool(tied))
    oc = ModelConfig.make(h, inter, layers, qh, kvh, hd, vocab, cap, tied=bool(tied))
    return g, qc, oc, cap


def _cos(a, b):
    a = bf(a).astype(np.float64).ravel()
    b = bf(b).astype(np.float64).ravel()
    return a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30)


@pytest.mark.parametrize("name", ["qwen3_0p6b", "qwen3_4b_l2", "qwen3_8b_l2", "qwen3_32b_l1"])
def test_prefill_then_decode_matches_oracle(oracle, name):
    from inference_b200 import Engine

    g, qc, oc, cap = _cfgs(name)
    toks = g["tokens"].astype(np.uint32)
    n = len(toks)
    n_pre = n - n // 3  # prefill two thirds, then decode the rest teacher-forced
    om = oracle.model(oc, seed=0)
    for t in toks[:n_pre]:
        om.forward(int(t))
    spread, ref_dev = spread_of(g, name)  # the reference's own implementations vs the oracle
    coss = []
    with Engine(qc, capacity=cap) as e:
        e.init_synthetic(0)
        e.set_tokens(toks)
        e.prefill(n_pre)
        e.sync()
        assert e.position == n_pre
        for i in range(n_pre):
            for lay in g["kv_layers"]:
                k, v = e.kv_slot(int(lay), i)
                ok_, ov_ = om.kv_slot(int(lay), i)
                assert _cos(k, ok_) >= 0.9995 and _cos(v, ov_) >= 0.9995, (i, int(lay))
                assert _cos(k, g[f"k_l{lay}"][i]) >= 0.999 and _cos(v, g[f"v_l{lay}"][i]) >= 0.999
        agree = 0
        for i in range(n_pre, n):
            e.step(1)
            e.sync()
            mine = e.logits()
            nxt = om.forward(int(toks[i]))
            coss.append(assert_within_spread(mine, om.logits(), spread)[1])
            agree += int(int(np.argmax(bf(mine))) == nxt)
        assert agree >= (n - n_pre) - 1
    om.close()
    paired_no_worse(1.0 - np.array(coss), ref_dev[n_pre:n])


def test_prefill_chunks_match_decode_steps():
    """A 700-token prompt prefills in two chunks (512 + 188 rows; the second
    chunk attends over the first one's cache); the cache and the next logits
    match the per-token decode path."""
    from inference_b200 import Engine, Qwen3Config, prompt_ids

    qc = Qwen3Config("qwen3-0.6b-l2", hidden=1024, inter=3072, layers=2, q_heads=16, kv_heads=8, vocab=151936,
                     tied=True)
    ids = prompt_ids(702)
    logits, kv = {}, {}
    for mode in ("prefill", "steps"):
        with Engine(qc, capacity=1024) as e:
            e.init_synthetic(0)
            e.set_tokens(ids)
            if mode == "prefill":
                e.prefill(700)
            else:
                e.step(700)
            e.step(1)
            e.sync()
            logits[mode] = e.logits()
            kv[mode] = {(lay, p): e.kv_slot(lay, p) for lay in (0, 1) for p in (0, 300, 511, 512, 699, 700)}
    for key, (k, v) in kv["steps"].items():
        kp, vp = kv["prefill"][key]
        assert _cos(k, kp) >= 0.9999 and _cos(v, vp) >= 0.9999, key
    assert_logits_close(logits["prefill"], logits["steps"], atol=3e-2, n_ulp=1, min_cos=0.9999)


def test_generate_uses_prefill_and_matches_steps():
    """q3_engine_generate (batched prefill + decode): every emitted token is the
    greedy choice of the per-token decode path fed the same sequence (up to a
    near-tie of the two fp32 orders: within 0.03 of the maximum logit)."""
    from inference_b200 import Engine, Qwen3Config, prompt_ids

    qc = Qwen3Config("qwen3-0.6b-l2", hidden=1024, inter=3072, layers=2, q_heads=16, kv_heads=8, vocab=151936,
                     tied=True)
    prompt = prompt_ids(40)
    n_new = 24
    with Engine(qc, capacity=128) as e:
        e.init_synthetic(0)
        out = np.asarray(e.generate(prompt, n_new, stop_at_eos=False))
        assert len(out) == n_new
        e.reset()
        e.set_tokens(np.concatenate([prompt, out]).astype(np.uint32))
        e.step(len(prompt) - 1)
        exact = 0
        for j in range(n_new):
            e.step(1)
            e.sync()
            lg = bf(e.logits()).astype(np.float64)
            assert lg[out[j]] >= lg.max() - 0.03, (j, lg[out[j]], lg.max())
            exact += int(int(np.argmax(lg)) == int(out[j]))
        assert exact >= n_new - 2
