"""NVFP4 weights on the GPU: the device quantizer + packed layout + dequantizer
bit-exact against the oracle's NVFP4 round trip, the NVFP4 GEMV against the
oracle's BF16 GEMV of the dequantized weights (exact BF16 values, so only the
fp32 summation order differs), and an NVFP4-weight engine against the oracle
model whose GEMV matrices are the same round trips (teacher forced, the BF16
engine's bounds)."""
import os

import numpy as np
import pytest

import make_golden as G
from gpu_util import assert_bf16_close, assert_within_spread, bf, dev, empty_bf16, host, paired_no_worse, spread_of
from inputs import uniform_bf16

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def be():
    from inference_b200 import B200Backend

    return B200Backend(0)


def _weights(seed, rows, cols):
    """BF16 rows spanning many binades, an all-zero row, blocks of zeros and a
    row whose blocks hit the E2M1 ties."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * np.exp2(rng.integers(-24, 10, (rows, 1)))).astype(np.float32)
    w[0] = 0.0
    if rows > 2:
        w[1, :32] = 0.0
        w[2, :16] = np.array([6, 5, 3.5, 2.5, 1.75, 1.25, 0.75, 0.25, -6, -5, -3.5, -2.5, -1.75, -1.25, -0.75, -0.25])
    return (w.view(np.uint32) >> 16).astype(np.uint16)


def _oracle_dequant(oracle, w):
    q, bs, rs = oracle.quantize_nvfp4(w)
    e2 = np.array([oracle.e2m1_value(c) for c in range(16)], np.float32)[q]
    s = np.array([oracle.e4m3_value(c) for c in range(256)], np.float32)[bs]
    deq = e2 * np.repeat(s, 16, axis=1) * rs[:, None]
    bits = (deq.view(np.uint32) >> 16).astype(np.uint16)
    assert np.array_equal(bf(bits), deq)  # exact BF16 values
    return bits, rs


@pytest.mark.parametrize("rows,cols", [(64, 1024), (37, 4096), (300, 12288), (8, 25600), (3, 64), (17, 2560)])
def test_quantize_roundtrip_matches_oracle_bit_exact(be, oracle, rows, cols):
    w = _weights(rows * 7 + cols, rows, cols)
    packed, rs = be.quantize_nvfp4(dev(w).view(rows, cols))
    back = be.dequant_nvfp4(packed, rs, rows, cols)
    obits, ors = _oracle_dequant(oracle, w)
    np.testing.assert_array_equal(host(rs), ors)
    np.testing.assert_array_equal(host(back), obits)


NVFP4_GEMV_SHAPES = [(1024, 151936), (4096, 6144), (4096, 24576), (12288, 4096), (25600, 5120), (2560, 19456),
                     (5120, 10240), (1536, 4096), (64, 3), (192, 1000), (3200, 777)]


@pytest.mark.parametrize("i,o", NVFP4_GEMV_SHAPES)
def test_gemv_nvfp4(be, oracle, i, o):
    x = uniform_bf16(G.seed_of("gemv4.x", i, o), (i,))
    w = uniform_bf16(G.seed_of("gemv4.w", i, o), (o, i))
    deq_bits, _ = _oracle_dequant(oracle, w)
    packed, rs = be.quantize_nvfp4(dev(w).view(o, i))
    y = empty_bf16(o)
    be.gemv_nvfp4(dev(x), packed, rs, y)
    assert_bf16_close(host(y), oracle.gemv(x, deq_bits), rtol=1e-2, atol=1e-3 * np.sqrt(i), min_exact=0.9)


def _cfgs(name):
    from inference_b200 import Qwen3Config
    from oracle import ModelConfig

    g = dict(np.load(os.path.join(GOLD, f"model_{name}_ref_cpu.npz")))
    h, inter, layers, qh, kvh, hd, vocab, cap, tied = (int(v) for v in g["config"])
    qc = Qwen3Config(name, hidden=h, inter=inter, layers=layers, q_heads=qh, kv_heads=kvh, vocab=vocab,
                     tied=bool(tied))
    oc = ModelConfig.make(h, inter, layers, qh, kvh, hd, vocab, cap, tied=bool(tied))
    return g, qc, oc, cap


@pytest.mark.parametrize("name", ["qwen3_0p6b", "qwen3_8b_l2", "qwen3_32b_l1"])
def test_nvfp4_engine_matches_nvfp4_oracle(oracle, name):
    from inference_b200 import Engine

    g, qc, oc, cap = _cfgs(name)
    toks = g["tokens"].astype(np.uint32)
    om = oracle.model(oc, seed=0).quantize_nvfp4()
    spread, ref_dev = spread_of(g, name)  # the reference's own implementations vs the oracle
    agree, coss = 0, []
    with Engine(qc, capacity=cap, weights="nvfp4") as e:
        e.init_synthetic(0)
        e.set_tokens(toks)
        for t in toks:
            e.step(1)
            e.sync()
            mine = e.logits()
            nxt = om.forward(int(t))
            coss.append(assert_within_spread(mine, om.logits(), spread)[1])
            agree += int(int(np.argmax(bf(mine))) == nxt)
        e.reset()
        out = e.generate(toks[:8], 4, stop_at_eos=False)
        assert len(out) == 4
    om.close()
    paired_no_worse(1.0 - np.array(coss), ref_dev[:len(coss)])
    assert agree >= len(toks) - 1


def test_nvfp4_engine_streams_about_a_quarter_of_the_weight_bytes():
    from inference_b200 import Engine, Qwen3Config

    qc = Qwen3Config("qwen3-tiny", hidden=1024, inter=3072, layers=2, q_heads=16, kv_heads=8, vocab=8192, tied=True)
    with Engine(qc, capacity=64) as a, Engine(qc, capacity=64, weights="nvfp4") as b:
        ratio = b.weight_bytes() / a.weight_bytes()
    assert 0.28 < ratio < 0.30, ratio
