"""Helpers for GPU tests: numpy BF16 bits <-> torch CUDA tensors, tolerances."""
from __future__ import annotations

import numpy as np


def torch():
    import torch as t

    return t


def dev(a: np.ndarray, dtype="bf16"):
    """uint16 BF16 bits (or float32) numpy -> CUDA tensor."""
    t = torch()
    if a.dtype == np.uint16:
        return t.from_numpy(np.ascontiguousarray(a).view(np.int16)).view(t.bfloat16).cuda()
    if a.dtype == np.float32:
        return t.from_numpy(np.ascontiguousarray(a)).cuda()
    if a.dtype in (np.int32, np.uint32):
        return t.from_numpy(np.ascontiguousarray(a).astype(np.int32)).cuda()
    raise TypeError(a.dtype)


def empty_bf16(*shape):
    t = torch()
    return t.empty(*shape, dtype=t.bfloat16, device="cuda")


def host(t_) -> np.ndarray:
    t = torch()
    t.cuda.synchronize()
    if t_.dtype == t.bfloat16:
        return t_.detach().cpu().view(t.int16).numpy().view(np.uint16)
    return t_.detach().cpu().numpy()


def bf(a: np.ndarray) -> np.ndarray:
    return (np.asarray(a, np.uint16).astype(np.uint32) << 16).view(np.float32)


def ulps(a, b):
    def key(x):
        x = np.asarray(x).astype(np.int32)
        return np.where(x & 0x8000, 0x8000 - (x & 0x7FFF), 0x8000 + x)
    return np.abs(key(a) - key(b))


def bf16_ulp(x):
    x = np.maximum(np.abs(np.asarray(x, np.float64)), 2.0 ** -126)
    return 2.0 ** (np.floor(np.log2(x)) - 7)


def assert_bf16_close(mine, gold, rtol=1e-2, atol=1e-2, min_exact=None, max_ulp=None):
    """The reference kernel tests' rule (rel 0.01 or abs margin per element,
    testing/util/tensor_matchers.hpp:55-62), plus optional ulp statistics."""
    m, g = bf(mine).astype(np.float64), bf(gold).astype(np.float64)
    bad = np.abs(m - g) > np.maximum(atol, rtol * np.abs(g))
    assert not bad.any(), f"{bad.sum()} mismatches, first at {np.argwhere(bad)[0]}: {m[bad][:4]} vs {g[bad][:4]}"
    d = ulps(mine, gold)
    if max_ulp is not None:
        assert d.max() <= max_ulp, f"max ulp distance {d.max()}"
    if min_exact is not None:
        assert (d == 0).mean() >= min_exact, f"exact fraction {(d == 0).mean():.4f}"


def assert_logits_close(mine, gold, atol=3e-2, n_ulp=2, min_cos=0.9999):
    """Model-level logits: |d| <= max(3e-2, 2 BF16 ulps) and cosine >= 0.9999."""
    m, g = bf(mine).astype(np.float64), bf(gold).astype(np.float64)
    bound = np.maximum(atol, n_ulp * bf16_ulp(g))
    bad = np.abs(m - g) > bound
    assert not bad.any(), f"{bad.sum()} logits off, e.g. {m[bad][:4]} vs {g[bad][:4]}"
    cos = m @ g / (np.linalg.norm(m) * np.linalg.norm(g) + 1e-30)
    assert cos >= min_cos, f"cosine {cos}"
    return float(np.abs(m - g).max()), float(cos)


def spread_of(g, name):
    """The reference's own implementation spread on a golden model record's
    steps: (max |logit difference| among the reference's implementations --
    its CPU backend vs the oracle, and, where tests/golden/make_golden_cuda.py
    has recorded it, its CUDA backend vs the oracle --, and per step the
    distance 1 - cosine of a GPU implementation of the reference from the
    oracle: its CUDA backend's where recorded, else its CPU backend's)."""
    import os

    spread = float(np.asarray(g["env_maxabs"]).max())
    dev = 1.0 - np.asarray(g["env_cos"], np.float64)
    p = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", f"model_{name}_ref_cuda.npz")
    if os.path.exists(p):
        c = np.load(p)
        spread = max(spread, float(np.asarray(c["cuda_maxabs"]).max()))
        dev = 1.0 - np.asarray(c["cuda_cos"], np.float64)
    return spread, dev


def assert_within_spread(mine, gold, spread):
    """Model-level logits held to a measured implementation spread, no scale
    factor: every |d| <= max(3e-2, spread) + one BF16 ulp of the gold logit (two
    results that differ by d in fp32 can round to BF16 values d + 1 ulp apart).
    Returns (max |d|, cosine) for the per-step comparison of paired_no_worse."""
    m, g = bf(mine).astype(np.float64), bf(gold).astype(np.float64)
    bound = max(3e-2, spread) + bf16_ulp(g)
    bad = np.abs(m - g) > bound
    assert not bad.any(), f"{bad.sum()} logits off, e.g. {m[bad][:4]} vs {g[bad][:4]} (spread {spread:.4f})"
    cos = m @ g / (np.linalg.norm(m) * np.linalg.norm(g) + 1e-30)
    return float(np.abs(m - g).max()), float(cos)


def paired_no_worse(mine, ref, what="1 - cosine"):
    """Per-step statistic of this implementation (e.g. 1 - cosine against the
    oracle) against the same statistic of the reference's own pair on the same
    steps: a paired one-sided test -- the mean difference stays within three
    standard errors of zero (it may be negative: closer than the reference)."""
    d = np.asarray(mine, np.float64) - np.asarray(ref, np.float64)
    se = d.std(ddof=1) / np.sqrt(len(d)) if len(d) > 1 else 0.0
    assert d.mean() <= 3.0 * se + 1e-12, (f"{what}: mean {np.mean(mine):.4g} vs the reference's {np.mean(ref):.4g} "
                                          f"(paired difference {d.mean():.3g}, 3 SE {3 * se:.3g})")
    return float(np.mean(mine)), float(np.mean(ref))
