"""The golden fixtures are the reference's own outputs, reproducibly.

tests/golden/make_golden.py generated them by running the reference's AVX-512
CPU backend and Qwen3 model (compiled from the reference's sources into
oracle/_ref/libref_cpu.so by oracle/build_ref.py).  Running the same generator
again must give back the committed arrays bit for bit: every kernel case, and
the whole Qwen3-0.6B teacher-forcing record (the reference's logits top-16,
greedy ids and KV slots, the oracle-vs-reference envelope).  The larger model
fixtures regenerate the same way (about a minute each, mostly synthetic
weights), so they are not part of this quick suite.
"""
import os

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = os.path.join(ROOT, "tests", "golden")
REF_CPU = os.path.join(ROOT, "oracle", "_ref", "libref_cpu.so")


@pytest.fixture(scope="module")
def refcpu():
    if not os.path.exists(REF_CPU):
        pytest.skip("reference CPU backend not built (oracle/build_ref.py needs the reference tree)")
    from oracle import RefLib

    return RefLib("cpu")


def _same(new, path):
    old = dict(np.load(path))
    assert set(new) == set(old), sorted(set(new) ^ set(old))
    bad = [k for k in sorted(new) if not np.array_equal(new[k], old[k])]
    assert not bad, f"fixtures that no longer reproduce: {bad[:8]}"


def test_kernel_fixtures_reproduce(refcpu):
    import make_golden as G

    _same(G.kernel_cases(refcpu), os.path.join(GOLD, "ops_ref_cpu.npz"))


@pytest.mark.slow
def test_qwen3_0p6b_fixture_reproduces(refcpu, oracle):
    import make_golden as G

    _same(G.model_case(refcpu, oracle, "qwen3_0p6b"), os.path.join(GOLD, "model_qwen3_0p6b_ref_cpu.npz"))
