"""FP8 E4M3 weights on the GPU: the device quantizer bit-exact against the
oracle's, the FP8 GEMV against the oracle's BF16 GEMV of the dequantized
weights (exact BF16 values, so only the fp32 summation order differs), and an
FP8-weight engine against the oracle model whose GEMV matrices are the same
E4M3 round trips (teacher forced, the BF16 engine's bounds)."""
import os

import numpy as np
import pytest

import make_golden as G
from gpu_util import assert_bf16_close, assert_logits_close, assert_within_spread, bf, dev, empty_bf16, host, paired_no_worse, spread_of
from inputs import uniform_bf16

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def be():
    from inference_b200 import B200Backend

    return B200Backend(0)


def _weights(seed, rows, cols):
    """BF16 rows spanning many binades, an all-zero row, and a row with a
    maximum of exactly 448 * 2^-3 (codes at the saturation edge)."""
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((rows, cols)) * np.exp2(rng.integers(-24, 10, (rows, 1)))).astype(np.float32)
    w[0] = 0.0
    if rows > 1:
        w[1] = rng.uniform(-40.0, 40.0, cols)
        w[1, cols // 2] = -56.0
    return (w.view(np.uint32) >> 16).astype(np.uint16)


def _torch_q(rows, cols):
    import torch

    return (torch.empty((rows, cols), dtype=torch.uint8, device="cuda"),
            torch.empty(rows, dtype=torch.float32, device="cuda"))


@pytest.mark.parametrize("rows,full,c0,cols", [(64, 1024, 0, 1024), (37, 4096, 1536, 512), (300, 12288, 0, 12288),
                                               (8, 25600, 6400, 6400), (3, 16, 2, 10)])
def test_quantize_matches_oracle_bit_exact(be, oracle, rows, full, c0, cols):
    w = _weights(rows * 7 + full, rows, full)
    q, sc = _torch_q(rows, cols)
    be.quantize_e4m3(dev(w).view(rows, full), q, sc, c0, cols)
    oq, osc = oracle.quantize_e4m3(w)  # scales from the full rows, as the device's
    np.testing.assert_array_equal(host(sc), osc)
    np.testing.assert_array_equal(host(q), oq[:, c0:c0 + cols])


# (in, out): Qwen3 shapes, tensor-parallel slices (3200 = 12.5 chunks of 256 columns), ragged
# row counts (partial 16-row tiles)
FP8_GEMV_SHAPES = [(1024, 151936), (4096, 6144), (4096, 24576), (12288, 4096), (25600, 5120), (2560, 19456),
                   (5120, 10240), (3200, 777), (1536, 4096), (64, 3), (192, 1000)]


@pytest.mark.parametrize("i,o", FP8_GEMV_SHAPES)
def test_gemv_e4m3(be, oracle, i, o):
    x = uniform_bf16(G.seed_of("gemv8.x", i, o), (i,))
    w = uniform_bf16(G.seed_of("gemv8.w", i, o), (o, i))
    oq, osc = oracle.quantize_e4m3(w)
    lut = np.array([oracle.e4m3_value(c) for c in range(256)], np.float32)
    deq = lut[oq] * osc[:, None]
    deq_bf = (deq.view(np.uint32) >> 16).astype(np.uint16)
    assert np.array_equal(bf(deq_bf), deq)  # exact BF16 values
    q, sc = _torch_q(o, i)
    import torch

    q.copy_(torch.from_numpy(oq))
    sc.copy_(torch.from_numpy(osc))
    y = empty_bf16(o)
    be.gemv_e4m3(dev(x), be.pack_e4m3(q), sc, y)
    mine = host(y)
    ref = oracle.gemv(x, deq_bf)
    assert_bf16_close(mine, ref, rtol=1e-2, atol=1e-3 * np.sqrt(i), min_exact=0.9)


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
def test_fp8_engine_matches_fp8_oracle(oracle, name):
    from inference_b200 import Engine

    g, qc, oc, cap = _cfgs(name)
    toks = g["tokens"].astype(np.uint32)
    om = oracle.model(oc, seed=0).quantize_fp8()
    spread, ref_dev = spread_of(g, name)  # the reference's own implementations vs the oracle
    agree, coss = 0, []
    with Engine(qc, capacity=cap, weights="fp8") as e:
        e.init_synthetic(0)
        e.set_tokens(toks)
        for t in toks:
            e.step(1)
            e.sync()
            mine = e.logits()
            nxt = om.forward(int(t))
            coss.append(assert_within_spread(mine, om.logits(), spread)[1])
            agree += int(int(np.argmax(bf(mine))) == nxt)
        # FP8 engines prefill through decode steps; generate still works
        e.reset()
        out = e.generate(toks[:8], 4, stop_at_eos=False)
        assert len(out) == 4
    om.close()
    paired_no_worse(1.0 - np.array(coss), ref_dev[:len(coss)])
    assert agree >= len(toks) - 1


def test_fp8_engine_streams_half_the_weight_bytes():
    from inference_b200 import Engine, Qwen3Config

    qc = Qwen3Config("qwen3-tiny", hidden=1024, inter=3072, layers=2, q_heads=16, kv_heads=8, vocab=8192, tied=True)
    with Engine(qc, capacity=64) as a, Engine(qc, capacity=64, weights="fp8") as b:
        ratio = b.weight_bytes() / a.weight_bytes()
    assert 0.5 < ratio < 0.52, ratio
