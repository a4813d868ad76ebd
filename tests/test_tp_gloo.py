"""Tensor-parallel decomposition on CPU with two gloo ranks.

Each rank generates only its shard of the weights (the same row/column
offsets the engine's q3_engine_init_synthetic uses), computes its partial
results with the oracle, and the ranks exchange them over gloo exactly as the
engine does over NCCL:
  * o_proj / down_proj are row-parallel: fp32 partial sums, allreduce(sum),
    then one BF16 rounding -- equal to the unsharded GEMV up to fp32 order;
  * gate/up are column shards, the SwiGLU output shard feeds down_proj;
  * lm_head is vocabulary-sharded: each rank's (value, global index) key is
    all-gathered and the maximum key wins -- the same first-index-of-maximum
    as the unsharded argmax, including ties across ranks.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _key(v: float, idx: int) -> int:
    b = np.array([v], np.float32).view(np.uint32)[0].item()
    b = (~b & 0xFFFFFFFF) if b & 0x80000000 else (b | 0x80000000)
    return (b << 32) | (0xFFFFFFFF - idx)


def _worker(rank, world, port, out_dir):
    import torch
    import torch.distributed as dist

    from oracle import Oracle, bf16_to_f32, f32_to_bf16

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    o = Oracle()
    H, I, qd_full, V = 256, 512, 512, 1024
    # o_proj: columns [rank*qd/N, ...) of the full [H, qd_full] matrix
    qd = qd_full // world
    x_full = o.normal(5, 900, 1, qd_full)[0]
    w_o_shard = o.normal(0, 19, H, qd, 0, rank * qd, qd_full)
    part = np.zeros(H, np.float32)
    xs = bf16_to_f32(x_full[rank * qd:(rank + 1) * qd])
    for j in range(H):
        part[j] = np.dot(bf16_to_f32(w_o_shard[j]).astype(np.float64), xs.astype(np.float64))
    t = torch.from_numpy(part)
    dist.all_reduce(t)
    o_tp = f32_to_bf16(t.numpy())
    # gate/up row shards + SwiGLU, then down_proj column shard
    il = I // world
    h_in = o.normal(6, 901, 1, H)[0]
    g = o.gemv(h_in, o.normal(0, 20, il, H, rank * il, 0, H))
    u = o.gemv(h_in, o.normal(0, 21, il, H, rank * il, 0, H))
    act = o.silu(g, u)
    acts = [torch.zeros(il, dtype=torch.int32) for _ in range(world)]
    dist.all_gather(acts, torch.from_numpy(act.astype(np.int32)))
    act_full = np.concatenate([a.numpy().astype(np.uint16) for a in acts])
    # lm_head vocabulary shard with a planted tie across the two ranks
    vl = V // world
    logits = o.gemv(h_in, o.normal(0, 22, vl, H, rank * vl, 0, H))
    if rank == 0:
        logits[vl - 3] = 0x4120  # 10.0 at global index vl-3
    else:
        logits[5] = 0x4120       # 10.0 at global index vl+5: the tie goes to the lower index
    lf = bf16_to_f32(logits)
    i_loc = int(np.argmax(lf))
    key = _key(float(lf[i_loc]), rank * vl + i_loc)
    k = torch.tensor([key - (1 << 64) if key >= (1 << 63) else key], dtype=torch.int64)
    keys = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
    dist.all_gather(keys, k)
    best = max(int(kk.item()) & 0xFFFFFFFFFFFFFFFF for kk in keys)
    greedy = 0xFFFFFFFF - (best & 0xFFFFFFFF)
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), o_tp=o_tp, act_full=act_full, greedy=greedy,
             logits=logits)
    dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_tensor_parallel_decomposition_two_gloo_ranks(tmp_path, oracle):
    from oracle import bf16_to_f32

    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, start_method="spawn")
    r0 = dict(np.load(tmp_path / "rank0.npz"))
    r1 = dict(np.load(tmp_path / "rank1.npz"))
    H, I, qd_full, V = 256, 512, 512, 1024
    # unsharded references
    x_full = oracle.normal(5, 900, 1, qd_full)[0]
    o_full = oracle.gemv(x_full, oracle.normal(0, 19, H, qd_full))
    np.testing.assert_array_equal(r0["o_tp"], r1["o_tp"])
    d = np.abs(bf16_to_f32(r0["o_tp"]) - bf16_to_f32(o_full))
    assert d.max() <= 2 * 2.0 ** (np.floor(np.log2(np.abs(bf16_to_f32(o_full)).max())) - 7)
    h_in = oracle.normal(6, 901, 1, H)[0]
    act = oracle.silu(oracle.gemv(h_in, oracle.normal(0, 20, I, H)), oracle.gemv(h_in, oracle.normal(0, 21, I, H)))
    np.testing.assert_array_equal(r0["act_full"], act)  # row shards: bit-identical to the full GEMV
    full_logits = np.concatenate([r0["logits"], r1["logits"]])
    assert int(r0["greedy"]) == int(r1["greedy"]) == oracle.argmax(full_logits) == V // 2 - 3
