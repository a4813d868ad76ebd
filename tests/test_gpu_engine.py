"""Model-level parity of the decode engine (CUDA graph path, through the C
ABI) against the oracle model and the reference's own CPU outputs.

Teacher forcing: both sides consume the same token sequence (the golden
fixture's prompt + the reference's greedy tokens), and every step's logits
are compared.  The bound per step is the larger of the stated target
(max |d| 3e-2, cosine 0.9999) and 1.5x the envelope that the reference's own
CPU backend and the oracle span over the run (stored in the fixture), or one BF16 ulp of the logit: two
correct fp32 implementations of a 2- or 28-layer random-weight Qwen3 already
land up to ~0.047 apart, so the kernels are held to "as close to the oracle
as the reference itself is".  Greedy argmax agreement >= 99% (here: all but
at most one step of a short run); KV-cache slots compared by direction.
"""
import os

import numpy as np
import pytest

from gpu_util import assert_within_spread, bf, paired_no_worse, spread_of

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
def test_engine_teacher_forced(oracle, name):
    from inference_b200 import Engine

    g, qc, oc, cap = _cfgs(name)
    toks = g["tokens"].astype(np.uint32)
    om = oracle.model(oc, seed=0)
    with Engine(qc, capacity=cap) as e:
        e.init_synthetic(0)
        e.set_tokens(toks)
        agree_oracle = agree_ref = 0
        worst, worst_cos = 0.0, 1.0
        mine_args, coss = [], []
        spread, ref_dev = spread_of(g, name)  # the reference's own implementations vs the oracle
        for i, t in enumerate(toks):
            e.step(1)
            e.sync()
            mine = e.logits()
            o_next = om.forward(int(t))
            ref = om.logits()
            d, c = assert_within_spread(mine, ref, spread)
            worst = max(worst, d)
            worst_cos = min(worst_cos, c)
            coss.append(c)
            # the reference's own logits at its top-16 indices
            ti = g["top_idx"][i]
            assert_within_spread(mine[ti], g["top_val"][i], spread)
            m_arg = int(np.argmax(bf(mine)))  # first index of the max, like the kernel
            mine_args.append(m_arg)
            agree_oracle += int(m_arg == o_next)
            agree_ref += int(m_arg == int(g["argmax"][i]))
            for lay in g["kv_layers"]:
                k, v = e.kv_slot(int(lay), i)
                ok_, ov_ = om.kv_slot(int(lay), i)
                assert _cos(k, ok_) >= 0.9995 and _cos(v, ov_) >= 0.9995
                assert _cos(k, g[f"k_l{lay}"][i]) >= 0.999 and _cos(v, g[f"v_l{lay}"][i]) >= 0.999
        hist = e.argmax_history(len(toks))
        np.testing.assert_array_equal(hist, mine_args)  # the fused lm_head argmax == argmax of its logits
    om.close()
    n = len(toks)
    paired_no_worse(1.0 - np.array(coss), ref_dev[:n])
    assert agree_oracle >= n - 1, (agree_oracle, n)
    assert agree_ref >= n - 1, (agree_ref, n)
    print(f"{name}: vs oracle max |dlogit| {worst:.4f} (reference CPU vs oracle: {g['env_maxabs'].max():.4f}), "
          f"min cosine {worst_cos:.6f} ({g['env_cos'].min():.6f}); argmax agreement oracle {agree_oracle}/{n}, "
          f"reference {agree_ref}/{n}")


def test_engine_argmax_history_and_forward_api(oracle):
    """q3_engine_forward (host round trip, Model::forward) and the device
    argmax history give the same greedy tokens as the kernels' logits."""
    from inference_b200 import Engine

    g, qc, oc, cap = _cfgs("qwen3_0p6b")
    toks = g["tokens"].astype(np.uint32)
    with Engine(qc, capacity=cap) as e:
        e.init_synthetic(0)
        nxt = []
        for t in toks[:12]:
            nxt.append(e.forward(int(t)))
            assert nxt[-1] == int(np.argmax(bf(e.logits())))
        e.reset()
        e.set_tokens(toks[:12])
        e.step(12)
        e.sync()
        hist = e.argmax_history(12)
        np.testing.assert_array_equal(hist, nxt)


def test_engine_generate_greedy_chain(oracle):
    """Generator::generate semantics: prompt prefill then greedy tokens; each
    generated token is the oracle's greedy choice given the same prefix."""
    from inference_b200 import QWEN3_0P6B, Engine, prompt_ids
    from oracle import ModelConfig

    cap = 48
    prompt = prompt_ids(16, seed=1)
    with Engine(QWEN3_0P6B, capacity=cap) as e:
        e.init_synthetic(0)
        out = e.generate(prompt, max_new=100)
        assert len(out) == cap - len(prompt)  # runs until the KV cache is full (generator.cpp:49)
        out2 = e.generate(prompt, max_new=8)
        np.testing.assert_array_equal(out2, out[:8])  # reset + regenerate is deterministic
    c = QWEN3_0P6B
    om = oracle.model(ModelConfig.make(c.hidden, c.inter, c.layers, c.q_heads, c.kv_heads, 128, c.vocab, cap,
                                       tied=True), seed=0)
    seq = list(prompt) + list(out)
    agree = 0
    for i in range(len(seq) - 1):
        nx = om.forward(int(seq[i]))
        if i >= len(prompt) - 1:
            agree += int(nx == int(seq[i + 1]))
    om.close()
    assert agree >= len(out) - 1


def test_engine_rejects_overflow():
    from inference_b200 import QWEN3_0P6B, Engine, Q3Error

    with Engine(QWEN3_0P6B.with_layers(1), capacity=8) as e:
        e.init_synthetic(0)
        e.set_tokens([1, 2, 3])
        e.step(8)
        e.sync()
        with pytest.raises(Q3Error):
            e.step(1)
        with pytest.raises(Q3Error):
            e.generate([1] * 8, max_new=4)


def test_batched_and_per_token_prefill_agree_at_long_context(oracle):
    """The batched prefill (tcgen05 GEMMs, batched attention) and the per-token
    decode steps over a 700-token prompt of a 4-layer Qwen3-0.6B (attention
    splits with several pages each), then 64 teacher-forced decode steps, each
    against the oracle: the batched path's mean max |d| and mean 1 - cosine over
    the steps are within 25% of the per-token path's, and the greedy choices
    agree but for near-ties (the two picks' logits closer than twice the
    paths' largest logit difference at that step).  The steps share one prompt's KV history, so they
    are not independent samples and a per-step paired test would be decided by
    that one history's rounding; the ratio bound holds both paths to the same
    error level instead."""
    from inference_b200 import QWEN3_0P6B, Engine, prompt_ids
    from oracle import ModelConfig

    cfg = QWEN3_0P6B.with_layers(4)
    seq = prompt_ids(700, seed=3)
    with Engine(cfg, capacity=1024) as e:
        e.init_synthetic(0)
        seq = np.concatenate([seq, e.generate(seq, max_new=64)])
    logits, args = {}, {}
    for mode in ("batched", "per_token"):
        with Engine(cfg, capacity=1024) as e:
            e.init_synthetic(0)
            e.set_tokens(seq)
            if mode == "batched":
                e.prefill(700)
            else:
                e.step(700)
            out = []
            for _ in range(64):
                e.step(1)
                e.sync()
                out.append(e.logits())
            logits[mode] = out
            args[mode] = e.argmax_history(764)[700:]
    om = oracle.model(ModelConfig.make(cfg.hidden, cfg.inter, cfg.layers, cfg.q_heads, cfg.kv_heads, 128, cfg.vocab,
                                       1024, tied=True), seed=0)
    for t in seq[:700]:
        om.forward(int(t))
    dev = {"batched": [], "per_token": []}
    for j in range(64):
        om.forward(int(seq[700 + j]))
        ref = bf(om.logits()).astype(np.float64)
        for mode in dev:
            m = bf(logits[mode][j]).astype(np.float64)
            dev[mode].append((np.abs(m - ref).max(), 1.0 - m @ ref / (np.linalg.norm(m) * np.linalg.norm(ref))))
    om.close()
    b, p = np.array(dev["batched"]), np.array(dev["per_token"])
    for col, what in ((0, "max |d|"), (1, "1 - cosine")):
        mb, mp = b[:, col].mean(), p[:, col].mean()
        assert mb <= 1.25 * mp, f"{what} vs the oracle: batched {mb:.4g}, per-token {mp:.4g}"
    # greedy choices: where the two paths pick different tokens, the batched path's
    # logits of the two picks lie within that step's batched-vs-per-token spread
    for j in np.nonzero(args["batched"] != args["per_token"])[0]:
        lb, lp = bf(logits["batched"][j]).astype(np.float64), bf(logits["per_token"][j]).astype(np.float64)
        gap = lb[args["batched"][j]] - lb[args["per_token"][j]]
        assert gap <= 2.0 * np.abs(lb - lp).max(), f"step {j}: a decisive greedy choice differs"
    assert (args["batched"] == args["per_token"]).mean() >= 0.9


def test_phase_timeline():
    """q3_engine_trace: one record per (CTA, launch) for the 5 launches of
    every layer and lm_head, in step order, and turning it off leaves the
    decoded tokens unchanged."""
    from inference_b200 import Engine, Qwen3Config, prompt_ids

    qc = Qwen3Config("qwen3-tiny", hidden=1024, inter=3072, layers=3, q_heads=16, kv_heads=8, vocab=8192, tied=True)
    ids = prompt_ids(24, vocab=qc.vocab)
    hist = {}
    for tracing in (False, True):
        with Engine(qc, capacity=256) as e:
            e.init_synthetic(0)
            e.set_tokens(ids[:8])
            if tracing:
                e.trace(True)
            e.step(16)
            e.sync()
            hist[tracing] = e.argmax_history(16)
            if tracing:
                raw = e.read_trace()
                e.trace(False)
                assert raw.shape[1] == 5 * qc.layers + 1 and raw.shape[2] == 10
                start, end = raw[..., 0].astype(np.int64), raw[..., 1].astype(np.int64)
                seen = start > 0
                assert seen.any(axis=0).all(), "every phase recorded"
                assert (end[seen] >= start[seen]).all()
                first = np.where(seen, start, np.iinfo(np.int64).max).min(axis=0)
                last_end = np.where(seen, end, 0).max(axis=0)
                assert (np.diff(first) >= 0).all(), "phases start in step order"
                assert last_end[-1] - first[0] < 10**8  # one step, well under 0.1 s
    np.testing.assert_array_equal(hist[False], hist[True])
