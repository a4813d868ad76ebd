"""Tensor-parallel engine on 2 GPUs (NCCL), teacher-forced against the oracle.

Each rank holds its head / MLP / vocabulary shard; the full logits are the
concatenation of the ranks' vocabulary shards and must match the oracle's
single-device model within the same envelope as the 1-GPU test; the greedy
argmax (resolved across ranks) must match the oracle's.
"""
import os
import socket

import numpy as np
import pytest

from gpu_util import assert_logits_close, bf

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, name, out_dir):
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
    e = Engine(qc, capacity=cap, device=rank, tp_rank=rank, tp_size=world)
    e.init_synthetic(0)
    obj = [Engine.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    e.attach_nccl(obj[0])
    e.set_tokens(toks)
    shards = []
    for _ in toks:
        e.step(1)
        e.sync()
        shards.append(e.logits())
    hist = e.argmax_history(len(toks))
    np.savez(os.path.join(out_dir, f"tp{rank}.npz"), logits=np.stack(shards), hist=hist)
    e.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(600)
@pytest.mark.parametrize("name", ["qwen3_8b_l2", "qwen3_0p6b"])
def test_engine_tensor_parallel_2gpu(tmp_path, oracle, name):
    import torch
    import torch.multiprocessing as mp

    from oracle import ModelConfig

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    mp.start_processes(_rank_main, args=(world, _free_port(), name, str(tmp_path)), nprocs=world,
                       start_method="spawn")
    parts = [dict(np.load(tmp_path / f"tp{r}.npz")) for r in range(world)]
    np.testing.assert_array_equal(parts[0]["hist"], parts[1]["hist"])  # every rank resolves the same token
    g = dict(np.load(os.path.join(GOLD, f"model_{name}_ref_cpu.npz")))
    h, inter, layers, qh, kvh, hd, vocab, cap, tied = (int(v) for v in g["config"])
    om = oracle.model(ModelConfig.make(h, inter, layers, qh, kvh, hd, vocab, cap, tied=bool(tied)), seed=0)
    atol = max(3e-2, 1.5 * float(g["env_maxabs"].max()))
    min_cos = min(0.9999, 1.0 - 1.5 * (1.0 - float(g["env_cos"].min())))
    agree = 0
    toks = g["tokens"]
    for i, t in enumerate(toks):
        nxt = om.forward(int(t))
        full = np.concatenate([parts[r]["logits"][i] for r in range(world)])
        assert_logits_close(full, om.logits(), atol=atol, n_ulp=1, min_cos=min_cos)
        assert int(parts[0]["hist"][i]) == int(np.argmax(bf(full)))
        agree += int(int(parts[0]["hist"][i]) == nxt)
    om.close()
    assert agree >= len(toks) - 1
