"""Parity against the reference's own CUDA backend (cuBLAS GEMV + its SIMT
kernels), built from the reference sources for sm_100a by oracle/build_ref.py
(oracle/_ref/libref_cuda.so), running on the same GPU.

Teacher-forced: the reference's CUDA and CPU Model::forward and the engine
consume the golden token sequence; per-step logits are compared, and the
reference's own CPU-vs-CUDA spread, measured on the same steps in the same
run, bounds the engine's distance from the reference CUDA backend.  The
full-depth, long-context version is tests/test_gpu_parity_full.py.
"""
import os

import numpy as np
import pytest

from gpu_util import assert_bf16_close, assert_within_spread, bf, dev, empty_bf16, host, paired_no_worse

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
    """The reference's CUDA and CPU backends and the engine consume the golden
    token sequence; the reference's own CPU-vs-CUDA spread on these steps bounds
    the engine's distance from the reference CUDA backend (plus one BF16 ulp of
    the output)."""
    from inference_b200 import Engine, Qwen3Config
    from oracle import ModelConfig, RefLib

    g = dict(np.load(os.path.join(GOLD, f"model_{name}_ref_cpu.npz")))
    h, inter, layers, qh, kvh, hd, vocab, cap, tied = (int(v) for v in g["config"])
    qc = Qwen3Config(name, hidden=h, inter=inter, layers=layers, q_heads=qh, kv_heads=kvh, vocab=vocab,
                     tied=bool(tied))
    mc = ModelConfig.make(h, inter, layers, qh, kvh, hd, vocab, cap, tied=bool(tied))
    rm = refcuda.model(mc, seed=0)
    cm = RefLib("cpu").model(mc, seed=0)
    toks = g["tokens"].astype(np.uint32)
    ref_logits, ref_next, ref_coss = [], [], []
    spread, ref_agree = 0.0, 0
    for t in toks:
        ref_next.append(rm.forward(int(t)))
        ref_logits.append(rm.logits())
        c_next = cm.forward(int(t))
        r, c = bf(ref_logits[-1]).astype(np.float64), bf(cm.logits()).astype(np.float64)
        spread = max(spread, float(np.abs(r - c).max()))
        ref_coss.append(float(r @ c / (np.linalg.norm(r) * np.linalg.norm(c))))
        ref_agree += int(c_next == ref_next[-1])
    rm.close()
    cm.close()
    worst, agree, coss = 0.0, 0, []
    with Engine(qc, capacity=cap) as e:
        e.init_synthetic(0)
        e.set_tokens(toks)
        for i in range(len(toks)):
            e.step(1)
            e.sync()
            mine = e.logits()
            d, c = assert_within_spread(mine, ref_logits[i], spread)
            worst = max(worst, d)
            coss.append(c)
            agree += int(int(np.argmax(bf(mine))) == ref_next[i])
    paired_no_worse(1.0 - np.array(coss), 1.0 - np.array(ref_coss))
    assert agree >= ref_agree - 1
    print(f"{name}: engine vs reference CUDA max |dlogit| {worst:.4f}, min cosine {min(coss):.6f}, argmax agreement "
          f"{agree}/{len(toks)}; reference CPU vs reference CUDA {spread:.4f}, {min(ref_coss):.6f}, "
          f"{ref_agree}/{len(toks)}")
