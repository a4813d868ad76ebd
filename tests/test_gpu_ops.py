"""Op-level parity of the sm_100a kernels (through the C ABI) against the
oracle and the reference's own outputs (tests/golden/ops_ref_cpu.npz).

Shapes: the reference's kernel tests (testing/tests/*.cpp) plus the Qwen3
decode shapes.  Tolerance: the reference's own rule, rel 0.01 per element
(testing/util/tensor_matchers.hpp), with an absolute margin for values near
zero, plus ulp statistics where the arithmetic is the same up to fp32 order.
"""
import numpy as np
import pytest

import make_golden as G
from gpu_util import assert_bf16_close, dev, empty_bf16, host, ulps
from inputs import uniform_bf16

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from inference_b200 import B200Backend

    return B200Backend(0)


GEMV_SHAPES = G.GEMV + [(1024, 151936), (4096, 6144), (4096, 24576), (12288, 4096), (25600, 5120), (9728, 2560),
                        (2560, 19456), (5120, 10240), (8, 3), (24, 1000)]


@pytest.mark.parametrize("i,o", GEMV_SHAPES)
def test_gemv(be, oracle, golden_ops, i, o):
    x = uniform_bf16(G.seed_of("gemv.x", i, o), (i,))
    w = uniform_bf16(G.seed_of("gemv.w", i, o), (o, i))
    y = empty_bf16(o)
    be.matmul(dev(x), dev(w), y)
    mine = host(y)
    ref = oracle.gemv(x, w)
    # same products, fp32 sums in another order: nearly all equal, the rest
    # one rounding apart (near-zero sums are bounded absolutely)
    assert_bf16_close(mine, ref, rtol=1e-2, atol=1e-3 * np.sqrt(i), min_exact=0.9)
    key = f"gemv/{i}x{o}"
    if key in golden_ops:
        assert_bf16_close(mine, golden_ops[key], rtol=1e-2, atol=1e-3 * np.sqrt(i), min_exact=0.9)


GEMM_SHAPES = [(1, 1024, 128), (130, 1024, 4096), (257, 2560, 1024), (512, 4096, 24576), (300, 12288, 4096)]


@pytest.mark.parametrize("m,k,n", GEMM_SHAPES)
def test_gemm_tcgen05(be, m, k, n):
    """Prefill GEMM (tcgen05, TMEM accumulator) against an fp32 product of the
    same BF16 operands; (512, 4096, 24576) runs the 256-column tile, the rest
    the 128-column tile, 130 / 257 / 300 rows exercise partial token tiles."""
    import torch

    x = uniform_bf16(G.seed_of("gemm.x", m, k, n), (m, k))
    w = uniform_bf16(G.seed_of("gemm.w", m, k, n), (n, k))
    y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    be.gemm(dev(x).view(m, k), dev(w).view(n, k), y)
    torch.cuda.synchronize()
    xf = dev(x).view(m, k).float()
    wf = dev(w).view(n, k).float()
    ref = (xf.double() @ wf.double().T).float().to(torch.bfloat16)
    mine = y.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
    gold = ref.view(torch.int16).cpu().numpy().view(np.uint16).reshape(-1)
    assert_bf16_close(mine, gold, rtol=1e-2, atol=1e-3 * np.sqrt(k), min_exact=0.9)


@pytest.mark.parametrize("h", G.NORM)
def test_rmsnorm(be, oracle, golden_ops, h):
    x = uniform_bf16(G.seed_of("norm.x", h), (h,))
    w = uniform_bf16(G.seed_of("norm.w", h), (h,))
    out = empty_bf16(h)
    be.rmsnorm(dev(x), dev(w), out, 1e-6)
    assert_bf16_close(host(out), golden_ops[f"rmsnorm/{h}"], max_ulp=1, min_exact=0.99)


@pytest.mark.parametrize("h", G.NORM)
def test_rmsnorm_add_aliased(be, golden_ops, h):
    """qwen3.hpp:152 passes the same tensor as update and output."""
    x = uniform_bf16(G.seed_of("norm.x", h), (h,))
    w = uniform_bf16(G.seed_of("norm.w", h), (h,))
    u = uniform_bf16(G.seed_of("norm.u", h), (h,))
    res, upd = dev(x), dev(u)
    be.rmsnorm_add(res, upd, dev(w), upd, 1e-6)
    np.testing.assert_array_equal(host(res), golden_ops[f"rmsnorm_add_res/{h}"])
    assert_bf16_close(host(upd), golden_ops[f"rmsnorm_add_out/{h}"], max_ulp=1, min_exact=0.99)


@pytest.mark.parametrize("qh,kvh,pos", G.QKNR)
def test_qk_norm_rope(be, oracle, golden_ops, qh, kvh, pos):
    q = uniform_bf16(G.seed_of("qknr.q", qh, kvh, pos), (qh, 128))
    k = uniform_bf16(G.seed_of("qknr.k", qh, kvh, pos), (kvh, 128))
    qn = uniform_bf16(G.seed_of("qknr.qn", qh, kvh, pos), (128,))
    kn = uniform_bf16(G.seed_of("qknr.kn", qh, kvh, pos), (128,))
    cache = be.make_rope_cache(pos + 1, 128, 1e6)
    qt, kt = dev(q), dev(k)
    be.qk_norm_rope(qt, kt, dev(qn), dev(kn), cache, pos, 1e-6)
    oq, ok = oracle.qk_norm_rope(q, k, qn, kn, pos)
    # oracle uses the same host RoPE tables: fp32 order differences only
    assert_bf16_close(host(qt), oq, atol=1e-2, min_exact=0.97)
    assert_bf16_close(host(kt), ok, atol=1e-2, min_exact=0.97)
    # the reference's tolerance against its own CPU outputs (qk_norm_rope.cpp:43-44)
    assert_bf16_close(host(qt), golden_ops[f"qknr_q/{qh}_{kvh}_{pos}"], atol=1e-2)
    assert_bf16_close(host(kt), golden_ops[f"qknr_k/{qh}_{kvh}_{pos}"], atol=1e-2)


# the last four have few kv heads and at least 16 pages: clusters of 16 splits where the
# GPU can hold one such cluster per kv head (the per-rank shapes of 4- and 8-way tensor
# parallelism), else 8
ATTN_CASES = G.ATTN + [(16, 8, 63), (16, 8, 64), (16, 8, 65), (32, 8, 127), (64, 8, 1000), (8, 8, 5), (16, 16, 200),
                       (32, 4, 700), (8, 1, 333), (64, 8, 8191), (8, 1, 2047), (8, 2, 4095), (2, 1, 1000), (1, 1, 1500)]


@pytest.mark.parametrize("qh,kvh,pos", ATTN_CASES)
def test_attention_reference_layout(be, oracle, golden_ops, qh, kvh, pos):
    q = uniform_bf16(G.seed_of("attn.q", qh, kvh, pos), (qh, 128))
    kc = uniform_bf16(G.seed_of("attn.k", qh, kvh, pos), (pos + 1, kvh, 128))
    vc = uniform_bf16(G.seed_of("attn.v", qh, kvh, pos), (pos + 1, kvh, 128))
    qt = dev(q)
    be.self_attention(qt, dev(kc), dev(vc), qt, pos)  # out aliases q (qwen3.hpp:149)
    mine = host(qt)
    assert_bf16_close(mine, oracle.attention(q, kc, vc, pos), rtol=1e-2, atol=2e-3)
    key = f"attn/{qh}_{kvh}_{pos}"
    if key in golden_ops:
        assert_bf16_close(mine, golden_ops[key], rtol=1e-2, atol=2e-3)


@pytest.mark.parametrize("qh,kvh,pos", [(16, 8, 0), (16, 8, 100), (32, 8, 4095), (64, 8, 2000), (8, 2, 64),
                                        (4, 1, 3000)])
def test_attention_paged_matches_flat(be, qh, kvh, pos):
    """The paged layout under a shuffled page table gives the same bits as the
    reference layout: the page table is only an address map."""
    q = uniform_bf16(G.seed_of("paged.q", qh, kvh, pos), (qh, 128))
    kc = uniform_bf16(G.seed_of("paged.k", qh, kvh, pos), (pos + 1, kvh, 128))
    vc = uniform_bf16(G.seed_of("paged.v", qh, kvh, pos), (pos + 1, kvh, 128))
    n_pages = pos // 64 + 1
    perm = np.random.default_rng(pos).permutation(n_pages + 3)[:n_pages].astype(np.int32)
    kp = np.zeros((n_pages + 3, kvh, 64, 128), np.uint16)
    vp = np.zeros_like(kp)
    for p in range(pos + 1):
        kp[perm[p // 64], :, p % 64] = kc[p]
        vp[perm[p // 64], :, p % 64] = vc[p]
    out_flat, out_paged = empty_bf16(qh, 128), empty_bf16(qh, 128)
    be.self_attention(dev(q), dev(kc), dev(vc), out_flat, pos)
    be.self_attention_paged(dev(q), dev(kp), dev(vp), dev(perm), out_paged, pos)
    np.testing.assert_array_equal(host(out_paged), host(out_flat))


@pytest.mark.parametrize("n", G.ELEM + [1 << 20])
def test_silu_and_add_aliased(be, oracle, golden_ops, n):
    a = uniform_bf16(G.seed_of("elem.a", n), (n,))
    b = uniform_bf16(G.seed_of("elem.b", n), (n,))
    g = dev(a)
    be.silu(g, dev(b), g)  # qwen3.hpp:156 aliases gate and output
    # CUDA expf and glibc expf may differ in the last fp32 bit: a BF16
    # rounding flip on at most a few elements per million
    d = ulps(host(g), oracle.silu(a, b))
    assert d.max() <= 1 and (d > 0).sum() <= max(1, n // 100000)
    l_ = dev(a)
    be.add(l_, dev(b), l_)  # qwen3.hpp:159 aliases left and output
    np.testing.assert_array_equal(host(l_), oracle.add(a, b))
    if f"silu/{n}" in golden_ops:
        assert ulps(host(g), golden_ops[f"silu/{n}"]).max() <= 1
        np.testing.assert_array_equal(host(l_), golden_ops[f"add/{n}"])


@pytest.mark.parametrize("n", G.ARGMAX)
def test_argmax(be, golden_ops, n):
    lg = uniform_bf16(G.seed_of("argmax", n), (n,))
    assert be.argmax(dev(lg)) == int(golden_ops[f"argmax/{n}"][0])


def test_argmax_ties_and_negatives(be, golden_ops):
    lg = uniform_bf16(G.seed_of("argmax.tie"), (4099,), -2.0, 1.0)
    lg[[17, 1000, 4098]] = 0x4040
    assert be.argmax(dev(lg)) == int(golden_ops["argmax_tie/4099"][0]) == 17
    neg = uniform_bf16(7, (151936,), -5.0, -1.0)
    neg[[5, 77777]] = 0xBF80  # -1.0 twice: the maximum, first index wins
    assert be.argmax(dev(neg)) == 5


def test_embedding(be, golden_ops):
    table = uniform_bf16(G.seed_of("embed"), (64, 1024))
    out = empty_bf16(1024)
    be.embedding(37, dev(table), out)
    np.testing.assert_array_equal(host(out), golden_ops["embedding/37"])


def test_fill_normal_matches_oracle(oracle):
    """Device weight generator == host generator, bit for bit (incl. shards)."""
    from inference_b200 import fill_normal

    t = __import__("torch")
    full = oracle.normal(0, 19, 300, 1000)
    d = t.empty(300 * 1000, dtype=t.bfloat16, device="cuda")
    fill_normal(d, 0, 19, 300, 1000)
    np.testing.assert_array_equal(host(d).reshape(300, 1000), full)
    shard = t.empty(100 * 250, dtype=t.bfloat16, device="cuda")
    fill_normal(shard, 0, 19, 100, 250, row0=50, col0=500, full_cols=1000)
    np.testing.assert_array_equal(host(shard).reshape(100, 250), full[50:150, 500:750])
    v = full.view(np.uint16)
    f = (v.astype(np.uint32) << 16).view(np.float32)
    assert abs(f.std() - 0.02) < 1e-3 and abs(f.mean()) < 1e-3

