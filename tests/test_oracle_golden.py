"""Pin the oracle (C restatement) against the reference's own outputs.

The fixtures under tests/golden/ were produced by the reference's AVX-512
CPU backend and Qwen3 model (tests/golden/make_golden.py).  Ops whose
arithmetic the oracle restates exactly must match bit for bit; ops where the
reference's -ffast-math build uses vectorised libm (exp, pow, cos, sin) must
match within one BF16 ulp on all but a handful of elements.
"""
import os

import numpy as np
import pytest

from inputs import bf16_to_f32, uniform_bf16
import make_golden as G

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def bf16_ulp(x):
    """Spacing of BF16 values at |x| (fp32 exponent, 8-bit significand)."""
    x = np.maximum(np.abs(np.asarray(x, np.float64)), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(x)) - 7)


def assert_logits_close(mine, gold, atol=3e-2, n_ulp=2):
    """|mine - gold| <= max(atol, n_ulp BF16 ulps of gold).  Logits are BF16,
    so above |x| = 4 a single rounding flip (0.031) already exceeds 3e-2."""
    mine = np.asarray(mine, np.float64)
    gold = np.asarray(gold, np.float64)
    bound = np.maximum(atol, n_ulp * bf16_ulp(gold))
    bad = np.abs(mine - gold) > bound
    assert not bad.any(), (mine[bad][:8], gold[bad][:8])


def ulps(a, b):
    """Distance in BF16 ulps (monotone integer mapping of the bit patterns)."""
    def key(x):
        x = x.astype(np.int32)
        return np.where(x & 0x8000, 0x8000 - (x & 0x7FFF), 0x8000 + x)
    return np.abs(key(a) - key(b))


@pytest.mark.parametrize("i,o", G.GEMV)
def test_gemv_exact(oracle, golden_ops, i, o):
    x = uniform_bf16(G.seed_of("gemv.x", i, o), (i,))
    w = uniform_bf16(G.seed_of("gemv.w", i, o), (o, i))
    np.testing.assert_array_equal(oracle.gemv(x, w), golden_ops[f"gemv/{i}x{o}"])


@pytest.mark.parametrize("h", G.NORM)
def test_rmsnorm_and_add_exact(oracle, golden_ops, h):
    x = uniform_bf16(G.seed_of("norm.x", h), (h,))
    w = uniform_bf16(G.seed_of("norm.w", h), (h,))
    u = uniform_bf16(G.seed_of("norm.u", h), (h,))
    np.testing.assert_array_equal(oracle.rmsnorm(x, w), golden_ops[f"rmsnorm/{h}"])
    res, out = oracle.rmsnorm_add(x, u, w)
    np.testing.assert_array_equal(res, golden_ops[f"rmsnorm_add_res/{h}"])
    np.testing.assert_array_equal(out, golden_ops[f"rmsnorm_add_out/{h}"])


@pytest.mark.parametrize("qh,kvh,pos", G.QKNR)
def test_qk_norm_rope(oracle, golden_ops, qh, kvh, pos):
    q = uniform_bf16(G.seed_of("qknr.q", qh, kvh, pos), (qh, 128))
    k = uniform_bf16(G.seed_of("qknr.k", qh, kvh, pos), (kvh, 128))
    qn = uniform_bf16(G.seed_of("qknr.qn", qh, kvh, pos), (128,))
    kn = uniform_bf16(G.seed_of("qknr.kn", qh, kvh, pos), (128,))
    q2, k2 = oracle.qk_norm_rope(q, k, qn, kn, pos)
    # The reference's cos/sin tables come from vectorised -ffast-math libm,
    # whose error grows with the angle (pos * inv_freq reaches ~8e3 rad); the
    # oracle's from scalar libm.  Nearly all elements agree to one ulp, and
    # all within the reference test's abs 0.01 (qk_norm_rope.cpp:43-44).
    for mine, key in ((q2, "qknr_q"), (k2, "qknr_k")):
        gold = golden_ops[f"{key}/{qh}_{kvh}_{pos}"]
        assert (ulps(mine, gold) <= 1).mean() >= 0.99
        np.testing.assert_allclose(bf16_to_f32(mine), bf16_to_f32(gold), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("qh,kvh,pos", G.ATTN)
def test_attention(oracle, golden_ops, qh, kvh, pos):
    q = uniform_bf16(G.seed_of("attn.q", qh, kvh, pos), (qh, 128))
    kc = uniform_bf16(G.seed_of("attn.k", qh, kvh, pos), (pos + 1, kvh, 128))
    vc = uniform_bf16(G.seed_of("attn.v", qh, kvh, pos), (pos + 1, kvh, 128))
    out = oracle.attention(q, kc, vc, pos)
    gold = golden_ops[f"attn/{qh}_{kvh}_{pos}"]
    # Same math, different fp32 summation order and exp implementation:
    # nearly every element is within one ulp; near-zero outputs (cancelling
    # weighted sums) are held to an absolute bound instead.
    assert (ulps(out, gold) <= 1).mean() >= 0.98
    np.testing.assert_allclose(bf16_to_f32(out), bf16_to_f32(gold), rtol=1e-2, atol=2e-3)


@pytest.mark.parametrize("n", G.ELEM)
def test_silu_add_exact(oracle, golden_ops, n):
    a = uniform_bf16(G.seed_of("elem.a", n), (n,))
    b = uniform_bf16(G.seed_of("elem.b", n), (n,))
    np.testing.assert_array_equal(oracle.silu(a, b), golden_ops[f"silu/{n}"])
    np.testing.assert_array_equal(oracle.add(a, b), golden_ops[f"add/{n}"])


@pytest.mark.parametrize("n", G.ARGMAX)
def test_argmax_exact(oracle, golden_ops, n):
    lg = uniform_bf16(G.seed_of("argmax", n), (n,))
    assert oracle.argmax(lg) == int(golden_ops[f"argmax/{n}"][0])


def test_argmax_ties_first_index(oracle, golden_ops):
    lg = uniform_bf16(G.seed_of("argmax.tie"), (4099,), -2.0, 1.0)
    lg[[17, 1000, 4098]] = 0x4040
    assert oracle.argmax(lg) == int(golden_ops["argmax_tie/4099"][0]) == 17


def test_embedding_exact(oracle, golden_ops):
    table = uniform_bf16(G.seed_of("embed"), (64, 1024))
    np.testing.assert_array_equal(oracle.embedding(37, table), golden_ops["embedding/37"])


def test_rope_tables(oracle, golden_ops):
    # The reference CPU build takes cos/sin through -ffast-math vectorised
    # libm, whose range reduction loses ~1e-4 at angles of a few thousand
    # radians; scalar libm (the oracle, and the reference's CUDA build, whose
    # host code has no -ffast-math) is accurate to ~1e-7.
    c, s = oracle.rope_cache(4096)
    rows = np.array([0, 1, 2, 511, 1023, 2047, 4095])
    np.testing.assert_allclose(c[rows], golden_ops["rope_cos_rows"], rtol=0, atol=5e-4)
    np.testing.assert_allclose(s[rows], golden_ops["rope_sin_rows"], rtol=0, atol=5e-4)


def _teacher_forced(oracle, name, max_steps=None):
    from oracle import ModelConfig

    g = dict(np.load(os.path.join(GOLD, f"model_{name}_ref_cpu.npz")))
    h, inter, layers, qh, kvh, hd, vocab, cap, tied = (int(v) for v in g["config"])
    cfg = ModelConfig.make(h, inter, layers, qh, kvh, hd, vocab, cap, tied=bool(tied))
    m = oracle.model(cfg, seed=0)
    toks = g["tokens"]
    n = len(toks) if max_steps is None else min(max_steps, len(toks))
    agree = 0
    for i in range(n):
        nxt = m.forward(int(toks[i]))
        lg = m.logits()
        f = bf16_to_f32(lg).astype(np.float64)
        gv = bf16_to_f32(g["top_val"][i]).astype(np.float64)
        # top-16 logits at the reference's top-16 indices
        assert_logits_close(f[g["top_idx"][i]], gv)
        # the sum of 151936 logits is mostly cancellation: bound it by the norm
        np.testing.assert_allclose(f.sum(), g["logit_sum"][i], rtol=0, atol=0.05 * np.sqrt(g["logit_sumsq"][i]))
        np.testing.assert_allclose((f * f).sum(), g["logit_sumsq"][i], rtol=1e-3)
        agree += int(nxt == int(g["argmax"][i]))
        for lay in g["kv_layers"]:
            k, v = m.kv_slot(int(lay), i)
            for mine, key in ((k, "k"), (v, "v")):
                gold = g[f"{key}_l{lay}"][i]
                # fp32-order differences compound over the layers below, so
                # deep-layer slots are compared by direction and a loose bound.
                a = bf16_to_f32(mine).astype(np.float64).ravel()
                b = bf16_to_f32(gold).astype(np.float64).ravel()
                assert a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30) >= 0.999
                assert np.abs(a - b).max() <= 0.15
    m.close()
    return agree, n


def test_model_0p6b_teacher_forced(oracle):
    agree, n = _teacher_forced(oracle, "qwen3_0p6b")
    assert agree >= n - 1


@pytest.mark.slow
@pytest.mark.parametrize("name", ["qwen3_4b_l2", "qwen3_8b_l2", "qwen3_32b_l1"])
def test_model_large_shapes_teacher_forced(oracle, name):
    agree, n = _teacher_forced(oracle, name)
    assert agree >= n - 1
