"""Parity against the reference's own CUDA backend (cuBLAS GEMV + its SIMT
kernels), built from the reference sources for sm_100a by oracle/build_ref.py
(oracle/_ref/libref_cuda.so), running on the same GPU.

Teacher-forced: the reference's CUDA Model::forward and the engine consume
the golden token sequence; per-step logits are compared.  Both sides now
carry their own fp32-order noise (each within the reference-CPU-vs-oracle
envelope of the fixture), so the bound is the sum of two envelopes: max
|d| <= max(3e-2, 2.5x envelope, one BF16 ulp), cosine >= 1 - 2.5 (1 - env).
The reference's own CUDA-vs-CPU spread is reported beside it.
"""
import os

import numpy as np
import pytest

from gpu_util import assert_bf16_close, assert_logits_close, bf, dev, empty_bf16, host

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")
REF_CUDA = os.path.join(ROOT, "oracle", "_ref", "libref_cuda.so")


@pytest.fixture(scope="module")
def refcuda():
    if not os.path.exists(REF_CUDA):
        pytest.skip("reference CUDA backend not built (oracle/build_ref.py needs the reference tree and CCCL 3.x)")
    import torch  # noqa: F401  (initialise the CUDA runtime first)

    from oracle import RefLib

    return RefLib("cuda")


def test_reference_cuda_ops_match(refcuda):
    """The reference's cuBLAS GEMV and flash-decode vs this library's kernels."""
    import make_golden as G
    from inputs import uniform_bf16

    from inference_b200 import B200Backend

    be = B200Backend(0)
    for i, o in [(1024, 2048), (4096, 6144), (4096, 24576), (12288, 4096), (1024, 151936)]:
        x = uniform_bf16(G.seed_of("rc.gemv.x", i, o), (i,))
        w = uniform_bf16(G.seed_of("rc.gemv.w", i, o), (o, i))
        y = empty_bf16(o)
        be.matmul(dev(x), dev(w), y)
        assert_bf16_close(host(y), refcuda.gemv(x, w), rtol=1e-2, atol=1e-3 * np.sqrt(i), min_exact=0.85)
    # Longest context first: the reference sizes its flash-attention scratch
    # once, from its first call's key length and query heads
    # (src/lib/backend/cuda/backend.cu:89-91,124-134); a later, longer call
    # would overflow it.  This library derives the split count per call.
    for qh, kvh, pos in [(32, 8, 4095), (32, 32, 1024), (16, 8, 777)]:
        q = uniform_bf16(G.seed_of("rc.attn.q", qh, kvh, pos), (qh, 128))
        kc = uniform_bf16(G.seed_of("rc.attn.k", qh, kvh, pos), (pos + 1, kvh, 128))
        vc = uniform_bf16(G.seed_of("rc.attn.v", qh, kvh, pos), (pos + 1, kvh, 128))
        out = empty_bf16(qh, 128)
        be.self_attention(dev(q), dev(kc), dev(vc), out, pos)
        assert_bf16_close(host(out), refcuda.attention(q, kc, vc, pos), rtol=1e-2, atol=2e-3)


@pytest.mark.parametrize("name", ["qwen3_0p6b", "qwen3_8b_l2"])
def test_engine_vs_reference_cuda_teacher_forced(refcuda, name):
    from inference_b200 import Engine, Qwen3Config
    from oracle import ModelConfig

    g = dict(np.load(os.path.join(GOLD, f"model_{name}_ref_cpu.npz")))
    h, inter, layers, qh, kvh, hd, vocab, cap, tied = (int(v) for v in g["config"])
    qc = Qwen3Config(name, hidden=h, inter=inter, layers=layers, q_heads=qh, kv_heads=kvh, vocab=vocab,
                     tied=bool(tied))
    rm = refcuda.model(ModelConfig.make(h, inter, layers, qh, kvh, hd, vocab, cap, tied=bool(tied)), seed=0)
    toks = g["tokens"].astype(np.uint32)
    atol = max(3e-2, 2.5 * float(g["env_maxabs"].max()))
    min_cos = min(0.9999, 1.0 - 2.5 * (1.0 - float(g["env_cos"].min())))
    worst = worst_ref = 0.0
    worst_cos = 1.0
    agree = 0
    with Engine(qc, capacity=cap) as e:
        e.init_synthetic(0)
        e.set_tokens(toks)
        for i, t in enumerate(toks):
            e.step(1)
            e.sync()
            mine = e.logits()
            r_next = rm.forward(int(t))
            ref = rm.logits()
            d, c = assert_logits_close(mine, ref, atol=atol, n_ulp=1, min_cos=min_cos)
            worst = max(worst, d)
            worst_cos = min(worst_cos, c)
            # the reference's own CUDA vs CPU spread at this step (top-16 of the CPU run)
            ti = g["top_idx"][i]
            worst_ref = max(worst_ref, float(np.abs(bf(ref[ti]) - bf(g["top_val"][i])).max()))
            agree += int(int(np.argmax(bf(mine))) == r_next)
    rm.close()
    assert agree >= len(toks) - 1
    print(f"{name}: engine vs reference CUDA max |dlogit| {worst:.4f}, min cosine {worst_cos:.6f}; "
          f"reference CUDA vs reference CPU "
          f"(top-16) {worst_ref:.4f}; argmax agreement {agree}/{len(toks)}")
