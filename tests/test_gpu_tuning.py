"""Determinism of the decode path (race detection) and the opt-in prefill
variants (q3_engine_set_tuning).

Every cross-CTA and cross-rank combination in the decode kernels runs in a
fixed order, so two independent runs on the same weights and ids must agree
bit for bit in every logit, argmax and KV slot -- on one GPU and across 2
tensor-parallel ranks.  The batched prefills of tensor-parallel and of
packed-weight engines change the fp32 order of the prefill's sums (GEMMs
instead of GEMVs, as the single-GPU prefill does), so they are held to the
oracle like test_gpu_prefill.py: KV slots of the prefilled positions and the
teacher-forced logits of the decode steps after it.
"""
import datetime
import os
import socket

import numpy as np
import pytest

from gpu_util import assert_logits_close, assert_within_spread, bf, paired_no_worse, spread_of

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")
TP_PREFILL = 0x10


def _cos(a, b):
    a = bf(a).astype(np.float64).ravel()
    b = bf(b).astype(np.float64).ravel()
    return a @ b / (np.linalg.norm(a) * np.linalg.norm(b) + 1e-30)


# GQA 4 with 2 kv heads (a small attention grid), Qwen3-0.6B and Qwen3-8B head and matrix shapes
@pytest.mark.parametrize("kv_heads,q_heads,hidden,inter", [(2, 8, 1024, 3072), (8, 16, 1024, 3072),
                                                           (8, 32, 4096, 12288)])
@pytest.mark.parametrize("weights", ["bf16", "fp8"])
def test_decode_is_deterministic(kv_heads, q_heads, hidden, inter, weights):
    """Race detection: two engines on the same weights and ids produce
    bit-identical logits, argmax and KV slots at every step, at positions from
    0 to the end of an 8192-slot cache (every page boundary the windows cross,
    up to 8 pages per split).  Every cross-CTA combination in the kernels is in
    a fixed order, so any difference is a race."""
    from inference_b200 import Engine, Qwen3Config, prompt_ids

    cfg = Qwen3Config(f"gqa{q_heads // kv_heads}-kv{kv_heads}-h{hidden}-l2", hidden=hidden, inter=inter, layers=2,
                      q_heads=q_heads, kv_heads=kv_heads, vocab=151936, tied=True)
    cap = 8192
    ids = prompt_ids(cap, seed=1)
    runs = {}
    for run in (0, 1):
        logits, kv = [], []
        with Engine(cfg, capacity=cap, weights=weights) as e:
            e.init_synthetic(0)
            e.set_tokens(ids)

            def window(n):
                for _ in range(n):
                    p = e.position
                    e.step(1)
                    e.sync()
                    logits.append(e.logits())
                    kv.append(e.kv_slot(1, p))

            window(70)         # positions 0..69: the first two pages, the live page the only one
            e.fill_kv(4090)    # synthetic cache: 64 pages, 4 per split
            window(10)         # 4090..4099 crosses the page boundary at 4096
            e.fill_kv(8180)
            window(11)         # 8180..8190: 128 pages, 8 per split
            hist = e.argmax_history(8191)
        runs[run] = (logits, kv, hist)
    base, tuned = runs[0], runs[1]
    for i, (a, b) in enumerate(zip(base[0], tuned[0])):
        assert np.array_equal(a, b), f"step {i}: logits differ"
    for i, ((k0, v0), (k1, v1)) in enumerate(zip(base[1], tuned[1])):
        assert np.array_equal(k0, k1) and np.array_equal(v0, v1), f"step {i}: KV slot differs"
    assert np.array_equal(base[2], tuned[2])


@pytest.mark.parametrize("name", ["qwen3_0p6b", "qwen3_8b_l2", "qwen3_32b_l1"])
def test_fp8_prefill_matches_fp8_oracle(oracle, name):
    """FP8 engine, batched prefill (each matrix expanded to its exact BF16 values,
    then the tcgen05 GEMMs), against the oracle's FP8 model fed token by token:
    the prefilled KV slots, then the teacher-forced logits of the decode steps."""
    from inference_b200 import Engine, Qwen3Config
    from oracle import ModelConfig

    g = dict(np.load(os.path.join(GOLD, f"model_{name}_ref_cpu.npz")))
    h, inter, layers, qh, kvh, hd, vocab, cap, tied = (int(v) for v in g["config"])
    qc = Qwen3Config(name, hidden=h, inter=inter, layers=layers, q_heads=qh, kv_heads=kvh, vocab=vocab,
                     tied=bool(tied))
    toks = g["tokens"].astype(np.uint32)
    n = len(toks)
    n_pre = n - n // 3
    om = oracle.model(ModelConfig.make(h, inter, layers, qh, kvh, hd, vocab, cap, tied=bool(tied)),
                      seed=0).quantize_fp8()
    for t in toks[:n_pre]:
        om.forward(int(t))
    spread, ref_dev = spread_of(g, name)  # the reference's own implementations vs the oracle
    coss = []
    with Engine(qc, capacity=cap, weights="fp8") as e:
        e.init_synthetic(0)
        e.tuning = ["fp8_prefill"]
        e.set_tokens(toks)
        e.prefill(n_pre)
        e.sync()
        assert e.position == n_pre
        for i in range(n_pre):
            for lay in g["kv_layers"]:
                k, v = e.kv_slot(int(lay), i)
                ok_, ov_ = om.kv_slot(int(lay), i)
                assert _cos(k, ok_) >= 0.9995 and _cos(v, ov_) >= 0.9995, (i, int(lay))
        agree = 0
        for i in range(n_pre, n):
            e.step(1)
            e.sync()
            mine = e.logits()
            nxt = om.forward(int(toks[i]))
            coss.append(assert_within_spread(mine, om.logits(), spread)[1])
            agree += int(int(np.argmax(bf(mine))) == nxt)
        assert agree >= (n - n_pre) - 1
    om.close()
    paired_no_worse(1.0 - np.array(coss), ref_dev[n_pre:n])


def test_tuning_rejects_unknown_bits():
    from inference_b200 import Engine, Q3Error, Qwen3Config

    cfg = Qwen3Config("qwen3-0.6b-l1", hidden=1024, inter=3072, layers=1, q_heads=16, kv_heads=8, vocab=151936,
                      tied=True)
    with Engine(cfg, capacity=64) as e:
        with pytest.raises(Q3Error):
            e.tuning = 0x400
        with pytest.raises(ValueError):
            e.tuning = ["no_such_flag"]
        for retired in (0x1, 0x2, 0x4, 0x8):
            with pytest.raises(Q3Error):
                e.tuning = retired
        e.tuning = ["all"]
        assert e.tuning == 0x30
        e.tuning = 0
        assert e.tuning == 0


# ---------------------------------------------------------------- 2 GPUs
def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _tp_main(rank, world, port, name, out_dir, mode, flags, n_pre):
    import torch
    import torch.distributed as dist

    from inference_b200 import Engine, Qwen3Config

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    g = dict(np.load(os.path.join(GOLD, f"model_{name}_ref_cpu.npz")))
    h, inter, layers, qh, kvh, hd, vocab, cap, tied = (int(v) for v in g["config"])
    qc = Qwen3Config(name, hidden=h, inter=inter, layers=layers, q_heads=qh, kv_heads=kvh, vocab=vocab,
                     tied=bool(tied))
    toks = g["tokens"].astype(np.uint32)
    e = Engine(qc, capacity=cap, device=rank, tp_rank=rank, tp_size=world)
    e.init_synthetic(0)
    e.tuning = flags
    if mode == "peer":
        hs = [None] * world
        dist.all_gather_object(hs, e.peer_handle())
        dist.barrier()  # every rank's buffer exists and is zeroed before anyone writes
        e.attach_peers(hs)
    else:
        obj = [Engine.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        e.attach_nccl(obj[0])
    e.set_tokens(toks)
    if n_pre:
        e.prefill(n_pre)
        e.sync()
    logits = []
    for _ in range(len(toks) - n_pre):
        e.step(1)
        e.sync()
        logits.append(e.logits())
    kv = {f"k{lay}_{p}": e.kv_slot(int(lay), p)[0] for lay in g["kv_layers"] for p in range(len(toks))}
    kv.update({f"v{lay}_{p}": e.kv_slot(int(lay), p)[1] for lay in g["kv_layers"] for p in range(len(toks))})
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), logits=np.stack(logits), hist=e.argmax_history(len(toks)),
             **kv)
    dist.barrier()  # no rank frees its exchange buffer while a peer may still use it
    e.close()
    dist.barrier()
    dist.destroy_process_group()


def _run_tp(tmp_path, tag, name, mode, flags, n_pre, world=2):
    import torch.multiprocessing as mp

    out = tmp_path / tag
    out.mkdir()
    mp.start_processes(_tp_main, args=(world, _free_port(), name, str(out), mode, flags, n_pre), nprocs=world,
                       start_method="spawn")
    return [dict(np.load(out / f"rank{r}.npz")) for r in range(world)]


@pytest.mark.timeout(600)
@pytest.mark.parametrize("name", ["qwen3_0p6b", "qwen3_8b_l2"])
def test_tp_decode_is_deterministic(tmp_path, name):
    """Two independent 2-rank runs (peer exchange): bit-identical on every rank."""
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    base = _run_tp(tmp_path, "base", name, "peer", 0, 0)
    tuned = _run_tp(tmp_path, "again", name, "peer", 0, 0)
    for r in range(2):
        for key in base[r]:
            assert np.array_equal(base[r][key], tuned[r][key]), (r, key)


@pytest.mark.timeout(600)
@pytest.mark.parametrize("mode", ["peer", "nccl"])
@pytest.mark.parametrize("name", ["qwen3_0p6b", "qwen3_8b_l2"])
def test_tp_prefill_matches_oracle(tmp_path, oracle, name, mode):
    import torch

    from oracle import ModelConfig

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    g = dict(np.load(os.path.join(GOLD, f"model_{name}_ref_cpu.npz")))
    h, inter, layers, qh, kvh, hd, vocab, cap, tied = (int(v) for v in g["config"])
    toks = g["tokens"]
    n = len(toks)
    n_pre = n - n // 3
    parts = _run_tp(tmp_path, "pf", name, mode, TP_PREFILL, n_pre, world)
    om = oracle.model(ModelConfig.make(h, inter, layers, qh, kvh, hd, vocab, cap, tied=bool(tied)), seed=0)
    kl = kvh // world
    for i in range(n_pre):
        om.forward(int(toks[i]))
        for lay in g["kv_layers"]:
            ok_, ov_ = om.kv_slot(int(lay), i)
            for r in range(world):
                k, v = parts[r][f"k{lay}_{i}"], parts[r][f"v{lay}_{i}"]
                assert _cos(k, ok_[r * kl:(r + 1) * kl]) >= 0.9995, (i, int(lay), r)
                assert _cos(v, ov_[r * kl:(r + 1) * kl]) >= 0.9995, (i, int(lay), r)
    spread, ref_dev = spread_of(g, name)  # the reference's own implementations vs the oracle
    agree, coss = 0, []
    for j, i in enumerate(range(n_pre, n)):
        nxt = om.forward(int(toks[i]))
        full = np.concatenate([parts[r]["logits"][j] for r in range(world)])
        coss.append(assert_within_spread(full, om.logits(), spread)[1])
        agree += int(int(np.argmax(bf(full))) == nxt)
    om.close()
    paired_no_worse(1.0 - np.array(coss), ref_dev[n_pre:n])
    assert agree >= (n - n_pre) - 1
