"""CPU-side checks of the C ABI: the library loads, exports every symbol
include/q3_sm100a.h declares, and rejects bad arguments before touching a
GPU.  No compute calls here."""
import ctypes as C
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    src = open(os.path.join(ROOT, "include", "q3_sm100a.h")).read()
    return sorted(set(re.findall(r"Q3_API\s+[\w\s\*]+?\b(q3_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from inference_b200 import lib
    from inference_b200._lib import SIGNATURES

    L = lib()
    syms = header_symbols()
    assert len(syms) >= 30
    for s in syms:
        assert hasattr(L, s), s
        assert s in SIGNATURES, f"{s} has no ctypes signature"
    assert set(SIGNATURES) == set(syms)


def test_invalid_arguments_fail_before_the_gpu():
    from inference_b200 import Q3Error, lib
    from inference_b200._lib import ModelConfig, check

    L = lib()
    assert L.q3_gemv(None, None, None, 4, 8, None) == 1
    assert b"null" in L.q3_last_error()
    x = C.c_void_p(16)  # never dereferenced: validation fails first
    assert L.q3_gemv(x, x, x, 4, 12, None) == 1  # n_in % 8
    assert L.q3_qk_norm_rope(x, x, x, x, x, x, 8, 8, 64, 0, 1e-6, None) == 3  # head_dim 64 unsupported
    assert L.q3_attention(x, x, x, x, 12, 8, 128, 5, x, 1 << 20, None) == 1  # 12 % 8
    bad = ModelConfig(1024, 3072, 28, 16, 8, 64, 151936, 1, 1e-6, 1e6, 64, 0)
    h = C.c_void_p()
    assert L.q3_engine_create(C.byref(bad), 0, 0, 1, C.byref(h)) == 3
    odd = ModelConfig(1024, 3072, 28, 16, 8, 128, 151936, 1, 1e-6, 1e6, 64, 0)
    assert L.q3_engine_create(C.byref(odd), 0, 0, 3, C.byref(h)) == 1  # 8 kv heads over 3 ranks
    assert L.q3_gemv_e4m3(x, x, x, x, 4, 24, None) == 1  # n_in % 16
    assert L.q3_engine_set_tuning(None, 0) == 1  # null engine
    flags = C.c_uint32(7)
    assert L.q3_engine_tuning(None, C.byref(flags)) == 1 and flags.value == 7
    assert L.q3_quantize_e4m3(x, 4, 64, 32, 48, x, x, None) == 1  # columns past the row
    assert L.q3_quantize_e4m3(x, 4, 64, 1, 8, x, x, None) == 1  # odd first column
    fmt = ModelConfig(1024, 3072, 28, 16, 8, 128, 151936, 1, 1e-6, 1e6, 64, 0, 7)
    assert L.q3_engine_create(C.byref(fmt), 0, 0, 1, C.byref(h)) == 1  # unknown weight format
    with pytest.raises(Q3Error):
        check(1)


def test_prompt_ids_and_rope_tables_match_oracle(oracle):
    from inference_b200 import prompt_ids, rope_tables

    np.testing.assert_array_equal(prompt_ids(4096, seed=1), oracle.prompt_ids(4096, seed=1))
    c1, s1 = rope_tables(8192)
    c2, s2 = oracle.rope_cache(8192)
    np.testing.assert_array_equal(c1, c2)
    np.testing.assert_array_equal(s1, s2)


def test_workspace_size_is_monotone():
    from inference_b200 import lib

    L = lib()
    sizes = [L.q3_attention_workspace_bytes(32, 8, p) for p in (0, 63, 64, 1000, 8191, 100000)]
    assert all(a <= b for a, b in zip(sizes, sizes[1:]))
    assert L.q3_attention_workspace_bytes(12, 8, 100) == 0


def test_drop_in_backend_harness_links_this_library():
    """oracle/_ref/libref_b200.so (the reference's Model and ops with the drop-in
    Backend of inference_b200/backend_b200/backend.cpp) loads without a GPU and
    resolves the C ABI to the in-tree libq3_sm100a.so."""
    path = os.path.join(ROOT, "oracle", "_ref", "libref_b200.so")
    if not os.path.exists(path):
        pytest.skip("drop-in backend harness not built (oracle/build_ref.py needs the reference tree)")
    L = C.CDLL(path)
    for s in ("ref_model_create", "ref_model_forward", "ref_model_logits", "ref_op_gemv", "ref_op_attention"):
        assert hasattr(L, s), s
    maps = open("/proc/self/maps").read()
    assert os.path.realpath(os.path.join(ROOT, "inference_b200", "libq3_sm100a.so")) in maps


def test_tuning_flag_names_match_the_header():
    """Engine.TUNE_FLAGS (names used by bench.py --tune) mirror the Q3_TUNE_* bits of
    include/q3_sm100a.h, and Q3_TUNE_ALL is their union."""
    from inference_b200 import Engine

    src = open(os.path.join(ROOT, "include", "q3_sm100a.h")).read()
    bits = {m.group(1).lower(): int(m.group(2), 16)
            for m in re.finditer(r"#define Q3_TUNE_(\w+) 0x([0-9A-Fa-f]+)u", src)}
    every = bits.pop("all")
    by_value = {v: k for k, v in bits.items()}
    assert sorted(Engine.TUNE_FLAGS.values()) == sorted(bits.values())
    for name, v in Engine.TUNE_FLAGS.items():
        assert name.replace("_", "") in by_value[v].replace("_", ""), (name, by_value[v])
    total = 0
    for v in bits.values():
        total |= v
    assert total == every


def test_tp_prefill_shard_shapes_fit_the_gemm():
    """Every Qwen3 configuration at every tensor-parallel size the engine accepts
    (kv heads, intermediate and vocabulary divisible by the ranks) gives shard
    GEMMs within the tcgen05 GEMM's shape rule (N % 128 == 0, K % 64 == 0;
    launch_gemm in gemm.cu), so Q3_TUNE_TP_PREFILL never meets a rejected shape."""
    from inference_b200.config import MODELS

    checked = 0
    for c in MODELS.values():
        for tp in (1, 2, 4, 8):
            if c.kv_heads % tp or c.inter % tp or (c.inter // tp) % 8 or c.vocab % tp:
                continue
            qd, kd, il, H = c.q_heads // tp * 128, c.kv_heads // tp * 128, c.inter // tp, c.hidden
            for n, k in ((qd + 2 * kd, H), (H, qd), (2 * il, H), (H, il)):
                assert n % 128 == 0 and k % 64 == 0, (c.name, tp, n, k)
            checked += 1
    assert checked == 16
