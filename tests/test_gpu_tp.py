"""Tensor-parallel engine on 2 GPUs, teacher-forced against the oracle, with
the partial sums exchanged by NCCL or through peer memory (CUDA IPC over
NVLink, fused into the GEMVs); one case with FP8 weights (against the
oracle's FP8 model: row-parallel shards keep their full rows' scales).

Each rank holds its head / MLP / vocabulary shard; the full logits are the
concatenation of the ranks' vocabulary shards and must match the oracle's
single-device model within the same envelope as the 1-GPU test; the greedy
argmax (resolved across ranks) must match the oracle's.
"""
import os
import socket

import numpy as np
import pytest

from gpu_util import assert_logits_close, assert_within_spread, bf, paired_no_worse, spread_of

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _attach(e, dist, mode, rank):
    from inference_b200 import Engine

    if mode == "peer":
        hs = [None] * dist.get_world_size()
        dist.all_gather_object(hs, e.peer_handle())
        dist.barrier()  # every rank's buffer exists and is zeroed before anyone writes
        e.attach_peers(hs)
    else:
        obj = [Engine.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        e.attach_nccl(obj[0])


def _rank_main(rank, world, port, name, out_dir, mode):
    import datetime

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
    exchange, _, weights = mode.partition("-")  # "peer-fp8": peer exchange, FP8 weights
    e = Engine(qc, capacity=cap, device=rank, tp_rank=rank, tp_size=world, weights=weights or "bf16")
    e.init_synthetic(0)
    _attach(e, dist, exchange, rank)
    e.set_tokens(toks)
    shards = []
    for _ in toks:
        e.step(1)
        e.sync()
        shards.append(e.logits())
    hist = e.argmax_history(len(toks))
    np.savez(os.path.join(out_dir, f"tp{rank}.npz"), logits=np.stack(shards), hist=hist)
    # peers read and write this rank's exchange buffer: every rank idle before any rank frees it
    e.sync()
    dist.barrier()
    e.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("name,mode,world", [("qwen3_8b_l2", "peer", 2), ("qwen3_8b_l2", "nccl", 2),
                                             ("qwen3_0p6b", "peer", 2), ("qwen3_0p6b", "nccl", 2),
                                             ("qwen3_8b_l2", "peer", 4), ("qwen3_0p6b", "peer-fp8", 2),
                                             ("qwen3_32b_l1", "peer", 2), ("qwen3_8b_l2", "peer", 8)])
def test_engine_tensor_parallel(tmp_path, oracle, name, mode, world):
    import torch
    import torch.multiprocessing as mp

    from oracle import ModelConfig

    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    mp.start_processes(_rank_main, args=(world, _free_port(), name, str(tmp_path), mode), nprocs=world,
                       start_method="spawn")
    parts = [dict(np.load(tmp_path / f"tp{r}.npz")) for r in range(world)]
    for r in range(1, world):
        np.testing.assert_array_equal(parts[0]["hist"], parts[r]["hist"])  # every rank resolves the same token
    g = dict(np.load(os.path.join(GOLD, f"model_{name}_ref_cpu.npz")))
    h, inter, layers, qh, kvh, hd, vocab, cap, tied = (int(v) for v in g["config"])
    om = oracle.model(ModelConfig.make(h, inter, layers, qh, kvh, hd, vocab, cap, tied=bool(tied)), seed=0)
    if mode.endswith("-fp8"):
        om.quantize_fp8()  # row scales over full rows: the same model as the 1-GPU FP8 engine
    spread, ref_dev = spread_of(g, name)  # the reference's own implementations vs the oracle
    agree, coss = 0, []
    toks = g["tokens"]
    for i, t in enumerate(toks):
        nxt = om.forward(int(t))
        full = np.concatenate([parts[r]["logits"][i] for r in range(world)])
        coss.append(assert_within_spread(full, om.logits(), spread)[1])
        assert int(parts[0]["hist"][i]) == int(np.argmax(bf(full)))
        agree += int(int(parts[0]["hist"][i]) == nxt)
    om.close()
    paired_no_worse(1.0 - np.array(coss), ref_dev[:len(coss)])
    assert agree >= len(toks) - 1


def _stall_main(rank, world, port, out_dir):
    import datetime

    import torch
    import torch.distributed as dist

    from inference_b200 import Engine, Q3Error, Qwen3Config, prompt_ids

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    qc = Qwen3Config("qwen3-0.6b-l2", hidden=1024, inter=3072, layers=2, q_heads=16, kv_heads=8, vocab=151936,
                     tied=True)
    e = Engine(qc, capacity=64, device=rank, tp_rank=rank, tp_size=world)
    e.init_synthetic(0)
    _attach(e, dist, "peer", rank)
    msg = ""
    if rank == 0:
        # rank 1 never steps: its flags never arrive, every wait must run out
        e.set_tokens(prompt_ids(4))
        e.step(1)
        try:
            e.sync()
        except Q3Error as exc:
            msg = str(exc)
        # the engine stays usable: its state reads back without error
        e.logits()
    dist.barrier()  # rank 1 keeps its buffer mapped until rank 0 is done
    with open(os.path.join(out_dir, f"stall{rank}.txt"), "w") as f:
        f.write(msg)
    e.close()
    dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_peer_wait_times_out_without_fault(tmp_path):
    """Failure detection: a peer that never produces its partials makes the
    bounded flag wait run out; the step reports Q3_ERR_DEVICE 'peer wait
    timed out' instead of hanging, and the context stays usable."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mp.start_processes(_stall_main, args=(2, _free_port(), str(tmp_path)), nprocs=2, start_method="spawn")
    msg = (tmp_path / "stall0.txt").read_text()
    assert "peer wait timed out" in msg, msg

