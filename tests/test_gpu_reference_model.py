"""The reference's own code running on this library.

oracle/_ref/libref_b200.so is the reference's Qwen3 Model and Backend ops
(src/lib/model/qwen3/qwen3.hpp, src/lib/backend/backend.hpp:16-42), compiled
from the reference sources by oracle/build_ref.py, with this repository's
drop-in Backend subclass (inference_b200/backend_b200/backend.cpp) linked in
place of the reference's CUDA backend -- the integration a maintainer makes.
The reference's Model, KVCache and Tensor code are unchanged; every op is a
call into libq3_sm100a.so.

Ops are held to the reference CPU backend's golden fixtures with the bounds of
test_gpu_ops.py.  Model::forward is teacher-forced against the oracle, within
twice the envelope between the reference's own CPU backend and the oracle (the
op-by-op path sums in fp32 orders of its own), with greedy agreement n - 1 or
better.
"""
import os

import numpy as np
import pytest

import make_golden as G
from gpu_util import assert_bf16_close, assert_logits_close, assert_within_spread, bf, paired_no_worse, spread_of, ulps
from inputs import uniform_bf16

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")
LIB = os.path.join(ROOT, "oracle", "_ref", "libref_b200.so")


def _cos(a, b):
    a = bf(a).astype(np.float64).ravel()
    b = bf(b).astype(np.float64).ravel()
    return a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30)


@pytest.fixture(scope="module")
def refb200():
    if not os.path.exists(LIB):
        pytest.skip("drop-in backend harness not built (oracle/build_ref.py needs the reference tree)")
    import torch  # noqa: F401  (initialise the CUDA runtime first)

    from oracle import RefLib

    return RefLib("b200")


def test_reference_ops_through_drop_in_backend(refb200, golden_ops):
    for i, o in G.GEMV:
        x = uniform_bf16(G.seed_of("gemv.x", i, o), (i,))
        w = uniform_bf16(G.seed_of("gemv.w", i, o), (o, i))
        assert_bf16_close(refb200.gemv(x, w), golden_ops[f"gemv/{i}x{o}"], rtol=1e-2, atol=1e-3 * np.sqrt(i),
                          min_exact=0.9)
    for h in G.NORM:
        x = uniform_bf16(G.seed_of("norm.x", h), (h,))
        w = uniform_bf16(G.seed_of("norm.w", h), (h,))
        u = uniform_bf16(G.seed_of("norm.u", h), (h,))
        assert_bf16_close(refb200.rmsnorm(x, w), golden_ops[f"rmsnorm/{h}"], max_ulp=1, min_exact=0.99)
        res, out = refb200.rmsnorm_add(x, u, w)
        np.testing.assert_array_equal(res, golden_ops[f"rmsnorm_add_res/{h}"])
        assert_bf16_close(out, golden_ops[f"rmsnorm_add_out/{h}"], max_ulp=1, min_exact=0.99)
    for qh, kvh, pos in G.QKNR:
        q = uniform_bf16(G.seed_of("qknr.q", qh, kvh, pos), (qh, 128))
        k = uniform_bf16(G.seed_of("qknr.k", qh, kvh, pos), (kvh, 128))
        qn = uniform_bf16(G.seed_of("qknr.qn", qh, kvh, pos), (128,))
        kn = uniform_bf16(G.seed_of("qknr.kn", qh, kvh, pos), (128,))
        oq, ok = refb200.qk_norm_rope(q, k, qn, kn, pos)
        assert_bf16_close(oq, golden_ops[f"qknr_q/{qh}_{kvh}_{pos}"], atol=1e-2)
        assert_bf16_close(ok, golden_ops[f"qknr_k/{qh}_{kvh}_{pos}"], atol=1e-2)
    for qh, kvh, pos in G.ATTN:
        q = uniform_bf16(G.seed_of("attn.q", qh, kvh, pos), (qh, 128))
        kc = uniform_bf16(G.seed_of("attn.k", qh, kvh, pos), (pos + 1, kvh, 128))
        vc = uniform_bf16(G.seed_of("attn.v", qh, kvh, pos), (pos + 1, kvh, 128))
        assert_bf16_close(refb200.attention(q, kc, vc, pos), golden_ops[f"attn/{qh}_{kvh}_{pos}"], rtol=1e-2,
                          atol=2e-3)
    for n in G.ELEM:
        a = uniform_bf16(G.seed_of("elem.a", n), (n,))
        b = uniform_bf16(G.seed_of("elem.b", n), (n,))
        if f"silu/{n}" in golden_ops:
            assert ulps(refb200.silu(a, b), golden_ops[f"silu/{n}"]).max() <= 1
            np.testing.assert_array_equal(refb200.add(a, b), golden_ops[f"add/{n}"])
    for n in G.ARGMAX:
        lg = uniform_bf16(G.seed_of("argmax", n), (n,))
        assert refb200.argmax(lg) == int(golden_ops[f"argmax/{n}"][0])
    table = uniform_bf16(G.seed_of("embed"), (64, 1024))
    np.testing.assert_array_equal(refb200.embedding(37, table), golden_ops["embedding/37"])


@pytest.mark.parametrize("name", ["qwen3_0p6b", "qwen3_8b_l2"])
def test_reference_model_on_drop_in_backend(refb200, oracle, name):
    from oracle import ModelConfig

    g = dict(np.load(os.path.join(GOLD, f"model_{name}_ref_cpu.npz")))
    h, inter, layers, qh, kvh, hd, vocab, cap, tied = (int(v) for v in g["config"])
    mc = ModelConfig.make(h, inter, layers, qh, kvh, hd, vocab, cap, tied=bool(tied))
    rm = refb200.model(mc, seed=0)
    om = oracle.model(mc, seed=0)
    spread, ref_dev = spread_of(g, name)  # the reference's own implementations vs the oracle
    agree, coss = 0, []
    toks = g["tokens"]
    for i, t in enumerate(toks):
        mine_next = rm.forward(int(t))  # Model::forward on the drop-in backend: greedy id via Backend::argmax
        ref_next = om.forward(int(t))
        mine = rm.logits()
        coss.append(assert_within_spread(mine, om.logits(), spread)[1])
        assert mine_next == int(np.argmax(bf(mine))), i
        agree += int(mine_next == ref_next)
        for lay in g["kv_layers"]:  # the KV slot Model::forward wrote through matmul + qk_norm_rope
            k, v = rm.kv_slot(int(lay), i)
            ok_, ov_ = om.kv_slot(int(lay), i)
            assert _cos(k, ok_) >= 0.999 and _cos(v, ov_) >= 0.999, (i, int(lay))
    rm.close()
    om.close()
    paired_no_worse(1.0 - np.array(coss), ref_dev[:len(coss)])
    assert agree >= len(toks) - 1
