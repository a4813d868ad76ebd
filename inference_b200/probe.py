"""Fixed kernel launches for profiling under ncu.

    python -m inference_b200.probe            # GEMV then prefill GEMM
    python -m inference_b200.probe attention  # decode attention
    python -m inference_b200.probe gemv8      # FP8-weight GEMV
    python -m inference_b200.probe decode [workload] [position] [steps]
    python -m inference_b200.probe timeline [workload] [position] [tune=a,b] [nccl]
    python -m torch.distributed.run --nproc-per-node N -m inference_b200.probe timeline ...

Default: three launches of the decode GEMV (q3_gemv, Qwen3-8B gate/up shape:
24576 x 4096, 201 MB of weights) followed by three launches of the prefill
GEMM (q3_gemm, 512 tokens x 4096 -> 24576) on cuda:0, random BF16 operands.
`attention`: three launches of the paged decode attention (q3_attention_paged)
for Qwen3-8B heads (32 q / 8 kv) at position 4095 with a 16-split cluster.
`gemv8`: the same gate/up shape with E4M3 weights (q3_quantize_e4m3 once,
then three q3_gemv_e4m3 launches), then the BF16 GEMV again; prints each
launch's CUDA-event time and GB/s (not meaningful under a profiler).
`decode`: decode steps of the CUDA-graph path (default qwen3-0.6b-ctx1024,
3 steps from position 520 over a synthetic KV cache); the only gemv_kernel /
attn_kernel launches of the process are those of the steps.
`timeline`: the CUDA-graph path's launch timeline (q3_engine_trace) of one
decode step at `position`, summarised per launch kind over layers 1..L-1:
CTA start to dependency release, prologue, main loop, epilogue (medians over
CTAs, microseconds), each launch's span from the previous launch's end, and
for tensor-parallel GEMVs the part of the prologue until every rank's partial
rows had arrived (`peers`).
Under torchrun the engine is tensor-parallel over the ranks (peer-memory
exchange, or NCCL with `nccl`) and every rank's summary is printed;
`tune=` applies q3_engine_set_tuning flags by name.
"""
import torch

from .backend import B200Backend


def attention():
    qh, kvh, pos = 32, 8, 4095
    pages = pos // 64 + 1
    be = B200Backend(0)
    q = torch.randn(qh, 128, device="cuda").to(torch.bfloat16)
    k = torch.randn(pages, kvh, 64, 128, device="cuda").to(torch.bfloat16)
    v = torch.randn(pages, kvh, 64, 128, device="cuda").to(torch.bfloat16)
    table = torch.arange(pages, dtype=torch.int32, device="cuda")
    out = torch.empty(qh, 128, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        be.self_attention_paged(q, k, v, table, out, pos)
    torch.cuda.synchronize()
    print("ok")


def gemv8():
    be = B200Backend(0)
    n, k = 24576, 4096
    x = torch.randn(k, device="cuda").to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda") * 0.02).to(torch.bfloat16)
    q = torch.empty(n, k, device="cuda", dtype=torch.uint8)
    sc = torch.empty(n, device="cuda", dtype=torch.float32)
    y = torch.empty(n, device="cuda", dtype=torch.bfloat16)
    be.quantize_e4m3(w, q, sc)
    q = be.pack_e4m3(q)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for name, fn, nbytes in (("fp8", lambda: be.gemv_e4m3(x, q, sc, y), n * k + 4 * n),
                             ("bf16", lambda: be.matmul(x, w, y), 2 * n * k)):
        for _ in range(3):
            flush.fill_(1)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            ms = a.elapsed_time(b)
            print(f"{name} {ms * 1000:.1f} us {nbytes / ms / 1e6:.0f} GB/s")
    print("ok")


def decode(workload="qwen3-0.6b-ctx1024", pos="520", steps="3"):
    from .config import WORKLOADS
    from .backend import prompt_ids
    from .engine import Engine

    cfg, _, cap = WORKLOADS[workload]
    pos, steps = int(pos), int(steps)
    with Engine(cfg, capacity=cap) as e:
        e.init_synthetic(0)
        e.persistent = False
        e.set_tokens(prompt_ids(16, vocab=cfg.vocab))
        e.fill_kv(pos)
        e.set_tokens(prompt_ids(pos + steps + 2, vocab=cfg.vocab))
        e.set_position(pos)
        e.step(steps)
        e.sync()
    print("ok")


def _tp_setup():
    """Under torchrun (WORLD_SIZE > 1): this rank's (rank, world, local device) and an
    initialised NCCL process group; (0, 1, 0, None) otherwise."""
    import datetime
    import os

    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world == 1:
        return 0, 1, 0, None
    import torch.distributed as dist

    rank, local = int(os.environ["RANK"]), int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return rank, world, local, dist


def timeline(workload="qwen3-0.6b-ctx1024", pos="520", *opts):
    """opts: tune=a,b (q3_engine_set_tuning names) and, under torchrun, nccl (the NCCL
    exchange instead of peer memory).  Each rank traces its own GPU (%globaltimer is
    per GPU); rank 0 prints every rank's summary in rank order."""
    import numpy as np

    from .backend import prompt_ids
    from .config import WORKLOADS
    from .engine import Engine

    cfg, _, cap = WORKLOADS[workload]
    pos = int(pos)
    tune = [t for o in opts if o.startswith("tune=") for t in o[5:].split(",") if t]
    rank, world, local, dist = _tp_setup()
    with Engine(cfg, capacity=cap, device=local, tp_rank=rank, tp_size=world) as e:
        e.init_synthetic(0)
        e.persistent = False
        if tune:
            e.tuning = tune
        if dist is not None:
            if "nccl" in opts:
                obj = [Engine.nccl_unique_id() if rank == 0 else None]
                dist.broadcast_object_list(obj, src=0)
                e.attach_nccl(obj[0])
            else:
                hs = [None] * world
                dist.all_gather_object(hs, e.peer_handle())
                dist.barrier()
                e.attach_peers(hs)
        e.set_tokens(prompt_ids(16, vocab=cfg.vocab))
        e.fill_kv(pos)
        e.set_tokens(prompt_ids(pos + 16, vocab=cfg.vocab))
        e.set_position(pos)
        e.step(4)
        e.trace(True)
        e.set_position(pos)
        e.step(3)
        e.sync()
        raw = e.read_trace().astype(np.float64)  # [ctas, phases, words]
        e.trace(False)
        if dist is not None:
            e.sync()
            dist.barrier()  # no rank frees its exchange buffer while a peer's last stores may target it
    seen = raw[..., 0] > 0
    t0, t1, c0, c1 = raw[..., 0], raw[..., 1], raw[..., 2], raw[..., 3]
    ghz = float(np.median(((c1 - c0) / np.maximum(t1 - t0, 1))[seen]))
    us = lambda cyc: cyc / ghz / 1e3
    n = raw.shape[1]
    ends = [t1[seen[:, k], k].max() for k in range(n)]
    lines = [f"{workload} position {pos} rank {rank}/{world}{' tuning ' + ','.join(tune) if tune else ''}: "
             f"step {(max(ends) - t0[seen].min()) / 1e3:.1f} us, SM clock {ghz:.3f} GHz"]
    names = ["qkv_gemv", "attention", "o_gemv", "gate_up_gemv", "down_gemv"]
    rows = {}
    for k in range(5, n - 1):
        v = seen[:, k]
        rows.setdefault(names[k % 5], []).append(
            [(ends[k] - ends[k - 1]) / 1e3, us(np.median(raw[v, k, 4])), us(np.median(raw[v, k, 5])),
             us(np.median(raw[v, k, 6])), us(np.median(raw[v, k, 7])), us(np.median(raw[v, k, 9]))])
    # peers: part of the prologue until thread 0 held every rank's partials (tensor parallel)
    lines.append(f"{'launch':14s} {'span':>7s} {'to_wait':>8s} {'prologue':>9s} {'loop':>7s} {'epilogue':>9s} "
                 f"{'peers':>7s}  (us)")
    for name in names:
        m = np.mean(rows[name], axis=0)
        lines.append(f"{name:14s} {m[0]:7.2f} {m[1]:8.2f} {m[2]:9.2f} {m[3]:7.2f} {m[4]:9.2f} {m[5]:7.2f}")
    v = seen[:, n - 1]
    lines.append(f"{'lm_head':14s} {(ends[n - 1] - ends[n - 2]) / 1e3:7.2f} {us(np.median(raw[v, n - 1, 4])):8.2f} "
                 f"{us(np.median(raw[v, n - 1, 5])):9.2f} {us(np.median(raw[v, n - 1, 6])):7.2f} "
                 f"{us(np.median(raw[v, n - 1, 7])):9.2f} {us(np.median(raw[v, n - 1, 9])):7.2f}")
    text = "\n".join(lines)
    if dist is None:
        print(text)
        return
    texts = [None] * world
    dist.all_gather_object(texts, text)
    if rank == 0:
        print("\n\n".join(texts))
    dist.barrier()
    dist.destroy_process_group()


def main():
    be = B200Backend(0)
    x = torch.randn(4096, device="cuda").to(torch.bfloat16)
    w = torch.randn(24576, 4096, device="cuda").to(torch.bfloat16)
    y = torch.empty(24576, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        be.matmul(x, w, y)
    xs = torch.randn(512, 4096, device="cuda").to(torch.bfloat16)
    ys = torch.empty(512, 24576, device="cuda", dtype=torch.bfloat16)
    for _ in range(3):
        be.gemm(xs, w, ys)
    torch.cuda.synchronize()
    print("ok")


if __name__ == "__main__":
    import sys

    {"attention": attention, "gemv8": gemv8, "decode": decode, "timeline": timeline}.get(sys.argv[1] if sys.argv[1:] else "", main)(*sys.argv[2:])
