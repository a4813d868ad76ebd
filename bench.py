"""Batch-1 Qwen3 decode benchmark (tokens/s and HBM roofline) on 1..8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

One bench step = one full greedy decode window of the workload: the cursor
is set back to the end of the prompt (prefilled once) and the engine decodes
to the context limit, (capacity - prompt) tokens, as Generator::generate's
loop does (src/lib/inference/generator.cpp:47-56, EOS ignored).  Weights are
synthetic N(0, 0.02) BF16 from seed 0, prompt ids uniform from seed 1.  With
N > 1 the model is tensor-parallel over N GPUs (strong scaling: the same
model and window, the work split by heads / MLP columns / vocabulary).

Rank 0 prints one JSON line.  `--impl reference` times the reference's own
CPU implementation (its AVX-512 backend compiled from its sources,
oracle/_ref/libref_cpu.so) on bounded samples of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "batch-1 decode tok/s and HBM GB/s vs roofline, 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--workload", default="qwen3-8b-ctx4096")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=0, help="profiling only: override the layer count")
    ap.add_argument("--window", type=int, default=0, help="profiling only: decode this many tokens per step")
    ap.add_argument("--prompt", type=int, default=0, help="profiling only: override the prompt length")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--nccl", action="store_true", help="tensor parallel: exchange partial sums with NCCL "
                    "instead of peer-memory stores fused into the GEMVs")
    ap.add_argument("--graph", action="store_true", help="use the per-step CUDA graph path (the default) even "
                                                          "where the persistent kernel was selected")
    ap.add_argument("--tune", default="", help="comma list of opt-in decode variants (q3_engine_set_tuning): "
                    "batched_poll, no_grid_wait, deep_ring, live_prefetch, tp_prefill, fp8_prefill, or all")
    ap.add_argument("--weights", default="bf16", choices=["bf16", "fp8"],
                    help="fp8: E4M3 GEMV matrices with per-row power-of-two scales (the FP8-weight model, "
                         "not the reference's BF16 model; the CUDA graph path)")
    ap.add_argument("--cpu-sample-tokens", type=int, default=3)
    ap.add_argument("--reference-cuda-tokens", type=int, default=0,
                    help="also time the reference's own cuBLAS CUDA backend (oracle/_ref/libref_cuda.so) for this "
                         "many Model::forward calls at mid-window context; reported as reference_cuda")
    ap.add_argument("--drop-in-tokens", type=int, default=0,
                    help="also time the reference's own Model::forward on this library's drop-in Backend "
                         "(oracle/_ref/libref_b200.so) for this many calls at mid-window context; reported as drop_in")
    return ap.parse_args()


def read_traffic_ratio(model_name):
    """DRAM bytes / algorithmic bytes of the dominant kernel, from the committed
    ncu summary profiles/traffic_<model>.md ("dram_bytes_per_algorithmic_byte: X")."""
    p = os.path.join(ROOT, "profiles", f"traffic_{model_name}.md")
    try:
        for line in open(p):
            if line.strip().startswith("dram_bytes_per_algorithmic_byte:"):
                return float(line.split(":", 1)[1])
    except OSError:
        pass
    return None


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def measured_bf16_peak():
    """Burst cuBLAS bf16 TFLOP/s of MEASURED_PEAKS.json (a prefill GEMM is timed alone)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return FALLBACK_BF16_TFLOPS, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_ids):
        self.gpu_ids = gpu_ids
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(prefix="clocks", suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={','.join(str(g) for g in self.gpu_ids)}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"], stdout=open(self.path, "w"),
                stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        rows = []
        try:
            for line in open(self.path):
                parts = [p.strip() for p in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except Exception:
            pass
        finally:
            try:
                os.unlink(self.path)
            except Exception:
                pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[1]) for r in rows if num(r[1]) is not None]
        mx = [num(r[2]) for r in rows if num(r[2]) is not None]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for name, val in zip(names, r[5:9]):
                if val.strip().lower() == "active":
                    reasons.add(name)
        load = [s for s in sm if s >= 0.5 * max(sm)] if sm else []
        return {"sm_mhz": statistics.median(load) if load else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(rows)}


# --------------------------------------------------------------------------- CPU legs
class CpuSampler:
    """The reference's own CPU backend (oracle/_ref/libref_cpu.so) -- or, where
    it was not built, the oracle's C port -- holding one model of the workload
    with its KV cache prefilled to context `pos` by synthetic values, timing
    Model::forward calls there."""

    def __init__(self, cfg, pos, max_tokens, threads):
        os.environ.setdefault("OMP_NUM_THREADS", str(threads))
        from oracle import ModelConfig

        mc = ModelConfig.make(cfg.hidden, cfg.inter, cfg.layers, cfg.q_heads, cfg.kv_heads, 128, cfg.vocab,
                              pos + max_tokens + 1, tied=cfg.tied)
        try:
            from oracle import RefLib

            impl, self.kind = RefLib("cpu"), "reference"
        except (FileNotFoundError, OSError):
            from oracle import Oracle

            impl, self.kind = Oracle(), "port"
        self.pos = pos
        self.m = impl.model(mc, seed=0)
        if self.kind == "reference":
            self.m.fill_kv(pos, seed=7)

    def sample(self, n_tokens):
        self.m.token_count = self.pos
        tok = 1000
        t0 = time.perf_counter()
        for _ in range(n_tokens):
            tok = self.m.forward(tok)
        return n_tokens / (time.perf_counter() - t0)

    def close(self):
        self.m.close()


def run_reference(a, cfg, prompt_len, capacity, workload):
    """--impl reference: the reference's CPU implementation, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    mid = prompt_len + (capacity - prompt_len) // 2
    n_tok = max(1, a.cpu_sample_tokens)
    cs = CpuSampler(cfg, mid, n_tok, threads)
    kind = cs.kind
    vals = [cs.sample(n_tok) for _ in range(a.warmup + a.steps)][a.warmup:]
    cs.close()
    value = statistics.mean(vals)
    sample = (f"{n_tok} decode steps (Model::forward) of {cfg.name} at context {mid} (mid-window of "
              f"{prompt_len}->{capacity}), KV cache prefilled with synthetic values, per bench step")
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tok/s", "n_gpus": a.gpus,
        "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(n_tok / value * 1000, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": workload, "model": cfg.name, "prompt": prompt_len, "context": capacity,
                   "global_batch": 1, "parallelism": "cpu", "l2_flush": "weights (GBs) exceed every cache"},
        "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": threads, "kind": kind,
                         "sample": sample},
        "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------- GPU leg
def main():
    a = parse_args()
    from inference_b200.config import WORKLOADS

    if a.workload not in WORKLOADS:
        raise SystemExit(f"unknown workload {a.workload}; choose from {sorted(WORKLOADS)}")
    cfg, prompt_len, capacity = WORKLOADS[a.workload]
    workload = a.workload
    if a.layers:
        cfg = cfg.with_layers(a.layers)
        workload += f"-L{a.layers}(profiling)"
    if a.prompt:
        prompt_len = a.prompt
        workload += f"-P{a.prompt}(profiling)"
    if a.window:
        workload += f"-W{a.window}(profiling)"
    if a.impl == "reference":
        return run_reference(a, cfg, prompt_len, capacity, workload)
    if a.warmup < 3:
        print("note: fewer than 3 warm-up steps", file=sys.stderr)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE {world}")
    import numpy as np
    import torch

    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    import inference_b200 as ib

    eng = ib.Engine(cfg, capacity=capacity, device=local, tp_rank=rank, tp_size=world, weights=a.weights)
    if a.weights == "fp8":
        workload += "-fp8"
    eng.init_synthetic(0)
    if a.graph and eng.persistent:
        eng.persistent = False
    tune = [t for t in a.tune.split(",") if t]
    if tune:
        eng.tuning = tune
        if "all" in tune:
            tune = sorted(ib.Engine.TUNE_FLAGS)
    if world > 1:
        if a.nccl:
            obj = [ib.Engine.nccl_unique_id() if rank == 0 else None]
            dist.broadcast_object_list(obj, src=0)
            eng.attach_nccl(obj[0])
        else:
            handles = [None] * world
            dist.all_gather_object(handles, eng.peer_handle())
            dist.barrier()  # every rank's exchange buffer exists and is zeroed before anyone writes
            eng.attach_peers(handles)

    window = capacity - prompt_len if not a.window else min(a.window, capacity - prompt_len)
    prompt = ib.prompt_ids(prompt_len, seed=1, vocab=cfg.vocab)
    stream = torch.cuda.ExternalStream(eng.stream(), device=torch.device("cuda", local))
    # prefill: every prompt id but the last (qwen3.hpp:168-173), batched through the
    # tcgen05 GEMMs; timed here (device events, max over ranks) and left in place
    pre_ms = []
    for rep_ in range(4):
        eng.reset()
        eng.set_tokens(prompt)
        p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        p0.record(stream)
        eng.prefill(prompt_len - 1)
        p1.record(stream)
        eng.sync()
        if rep_:
            pre_ms.append(p0.elapsed_time(p1))
    pre_t = float(np.median(pre_ms))
    if dist:
        t = torch.tensor([pre_t], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        pre_t = float(t.item())
    start_pos = prompt_len - 1

    def one_window():
        eng.set_position(start_pos)
        eng.step(window)

    def barrier():
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(a.warmup):
        one_window()
    eng.sync()
    barrier()

    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gpu_ids = list(range(world)) if world > 1 else [local]
    with ClockSampler(gpu_ids) as clocks:
        ev0.record(stream)
        for _ in range(a.steps):
            one_window()
        ev1.record(stream)
        eng.sync()
    ms = ev0.elapsed_time(ev1)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clock = clocks.summary()
    tokens = a.steps * window
    tok_s = tokens / (ms / 1000.0)

    # ---- end-to-end through the public API (host buffers, H2D + D2H inside)
    e2e = None
    if not a.no_e2e:
        pin_prompt = torch.from_numpy(prompt.astype(np.int32)).pin_memory()
        pin_out = torch.empty(window, dtype=torch.int32).pin_memory()
        import ctypes as C

        n_out = C.c_size_t()
        barrier()
        t0 = time.perf_counter()
        for _ in range(a.steps):
            ib._lib.check(ib.lib().q3_engine_generate(eng.h, pin_prompt.data_ptr(), prompt_len, window, 0,
                                                      pin_out.data_ptr(), C.byref(n_out)))
        torch.cuda.synchronize()
        dt = time.perf_counter() - t0
        if dist:
            t = torch.tensor([dt], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            dt = float(t.item())
        e2e = {"value": round(a.steps * window / dt, 3), "unit": "tok/s", "h2d_bytes_per_step": int(prompt_len * 4 + 4),
               "d2h_bytes_per_step": int(window * 4),
               "includes": "prompt H2D, prefill of the prompt, decode, token D2H"}

    # ---- prefill (informational: the metric is decode tok/s)
    n_pre = prompt_len - 1
    # every layer's four GEMMs, but the last layer stops after its QKV GEMM
    gemm_flop = 2.0 * n_pre * (cfg.layer_matmul_params() * (cfg.layers - 1) +
                               (cfg.q_heads + 2 * cfg.kv_heads) * cfg.head_dim * cfg.hidden)
    attn_flop = 4.0 * cfg.layers * cfg.q_heads * cfg.head_dim * n_pre * (n_pre + 1) / 2.0
    bf16_peak, bf16_kind = measured_bf16_peak()
    prefill = {"tokens": n_pre, "ms": round(pre_t, 3), "tok_s": round(n_pre / (pre_t / 1000.0), 1),
               "path": ("batched: tcgen05 GEMMs (TMEM accumulators, TMA), batched split-KV attention"
                        + ("; row-parallel fp32 partials exchanged between ranks" if world > 1 else "")
                        + ("; E4M3 matrices expanded to their BF16 values first" if a.weights == "fp8" else "")
                        if (a.weights == "bf16" or "fp8_prefill" in tune) and (world == 1 or "tp_prefill" in tune)
                        else "per-token decode steps"),
               "tflops": round((gemm_flop + attn_flop) / (pre_t / 1000.0) / 1e12 / world, 1),
               "gemm_tflop": round(gemm_flop / 1e12, 3), "attention_tflop": round(attn_flop / 1e12, 3),
               "peak_tflops": bf16_peak, "frac": round((gemm_flop + attn_flop) / (pre_t / 1000.0) / 1e12 / world /
                                                      bf16_peak, 4),
               "peak_kind": bf16_kind}

    # ---- dominant kernel roofline
    peak, peak_kind = measured_peaks()
    avg_pos = start_pos + (window - 1) / 2.0
    bytes_tok = cfg.weight_bytes(a.weights) + cfg.kv_bytes_per_position() * (avg_pos + 1)
    mid = start_pos + window // 2
    # the kernel-per-op path, one eager step with CUDA events around each launch (diagnostic)
    eng.set_position(mid)
    g_ms, g_launch, g_bytes = eng.profile_step(0)
    eng.set_position(mid)
    at_ms, at_launch, at_bytes = eng.profile_step(1)
    eager = {"gemv_gbs": round(g_bytes / (g_ms / 1000.0) / 1e9, 1), "gemv_launch_ms_avg": round(g_ms / g_launch, 5),
             "gemv_launches_per_step": g_launch,
             "attention_gbs": round(at_bytes / (at_ms / 1000.0) / 1e9, 1),
             "attention_launch_ms_avg": round(at_ms / max(1, at_launch), 5)}
    traffic_ratio = read_traffic_ratio(cfg.name)
    if eng.persistent:
        # one cooperative launch per bench step: algorithmic bytes of the whole window / its device time
        per_launch = bytes_tok * window / world
        achieved = bytes_tok * tok_s / 1e9 / world
        roofline = {"kernel": "persistent_decode_kernel (one cooperative launch = one decode window of "
                              f"{window} tokens)",
                    "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                    "traffic": round(traffic_ratio * per_launch) if traffic_ratio else None,
                    "algorithmic_bytes_per_launch": round(per_launch), "launch_ms_avg": round(ms / a.steps, 3),
                    "kernel_per_op_path": eager}
        launches = a.steps
    else:
        achieved = g_bytes / (g_ms / 1000.0) / 1e9
        roofline = {"kernel": "gemv_kernel (every GEMV launch of one decode step; per-launch averages)",
                    "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                    "traffic": round(traffic_ratio * g_bytes / g_launch) if traffic_ratio else None,
                    "algorithmic_bytes_per_launch": round(g_bytes / g_launch),
                    "launch_ms_avg": round(g_ms / g_launch, 5), "launches_per_step": g_launch,
                    "kernel_per_op_path": eager}
        launches = (cfg.layers * 5 + 1) * window * a.steps
    # whole-step roofline: weights + average KV read per token over the window, all ranks
    step_roof = {"bytes_per_token": int(bytes_tok), "achieved_gbs": round(bytes_tok * tok_s / 1e9, 1),
                 "peak_gbs": peak * world, "frac": round(bytes_tok * tok_s / 1e9 / (peak * world), 4)}

    # ---- CPU baseline (rank 0, N = 1 only)
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        threads = os.cpu_count() or 1
        try:
            cs = CpuSampler(cfg, mid, a.cpu_sample_tokens, threads)
            cs.sample(1)
            v, kind = cs.sample(a.cpu_sample_tokens), cs.kind
            cs.close()
            cpu = {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": kind,
                   "sample": f"{a.cpu_sample_tokens} decode steps of {cfg.name} at context {mid}, KV prefilled "
                             f"with synthetic values"}
        except Exception as exc:  # report, never fail the GPU number
            cpu = {"value": None, "unit": "tok/s", "cores": threads, "kind": "reference", "sample": f"failed: {exc}"}

    # ---- the reference's own Model::forward on the same GPU (optional, rank 0, N = 1):
    # with its cuBLAS CUDA backend, and with this library's drop-in Backend
    timed_refs = {}
    for key, kind, n_req, what in (("reference_cuda", "cuda", a.reference_cuda_tokens,
                                    "reference cuBLAS CUDA backend built from its sources for sm_100a"),
                                   ("drop_in", "b200", a.drop_in_tokens,
                                    "the reference's Model::forward on this library's drop-in Backend "
                                    "(inference_b200/backend_b200/backend.cpp)")):
        if not (rank == 0 and world == 1 and n_req > 0):
            continue
        try:
            from oracle import ModelConfig, RefLib

            rl = RefLib(kind)
            n_tok = n_req
            mc = ModelConfig.make(cfg.hidden, cfg.inter, cfg.layers, cfg.q_heads, cfg.kv_heads, 128, cfg.vocab,
                                  mid + n_tok + 2, tied=cfg.tied)
            rm = rl.model(mc, seed=0)
            rm.fill_kv(mid, seed=7)
            rm.forward(1000)  # the first call allocates the backend's scratch (the reference's flash scratch)
            rm.token_count = mid
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            tok = 1000
            for _ in range(n_tok):
                tok = rm.forward(tok)  # Model::forward: host sync per token, as the reference generator runs
            dt = time.perf_counter() - t0
            rm.close()
            timed_refs[key] = {"value": round(n_tok / dt, 3), "unit": "tok/s",
                               "sample": f"{n_tok} Model::forward calls at context {mid}, {what}"}
        except Exception as exc:
            timed_refs[key] = {"value": None, "unit": "tok/s", "sample": f"failed: {exc}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(tok_s, 3), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": workload, "model": cfg.name, "prompt": prompt_len, "context": capacity,
                       "decode_tokens_per_step": window, "global_batch": 1,
                       "decode_path": "persistent kernel" if eng.persistent else "CUDA graph of fused kernels",
                       "parallelism": f"tp{world}", "weight_format": a.weights, "tuning": tune,
                       "tp_exchange": (None if world == 1 else "NCCL allreduce/allgather" if a.nccl else
                                       "peer-memory stores fused into the o/down/lm_head GEMVs (CUDA IPC, NVLink)"), "weights": "random N(0,0.02) seed 0, ids seed 1",
                       "l2_flush": f"not needed: {cfg.weight_bytes(a.weights) / 1e9:.1f} GB of weights streamed per token "
                                   f">> 126 MB L2"},
            "clocks": clock, "e2e": e2e, "gpu_launches": int(launches),
            "roofline": roofline, "step_roofline": step_roof, "cpu_baseline": cpu, "prefill": prefill,
        }
        line.update(timed_refs)
        print(json.dumps(line), flush=True)
    if dist:
        # a rank's last kernels store into its peers' exchange buffers: every rank's
        # stream is idle before any rank frees its buffer
        eng.sync()
        dist.barrier()
    eng.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
