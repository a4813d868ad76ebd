"""Batch-1 Qwen3 decode benchmark (tokens/s and HBM roofline) on 1..8 B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...
    python bench.py --probe gemv|attention|gemv8|decode|timeline [...]   (fixed launches for ncu, timelines)

One bench step = one full greedy decode window of the workload: the cursor
is set back to the end of the prompt (prefilled once) and the engine decodes
to the context limit, (capacity - prompt) tokens, as Generator::generate's
loop does (src/lib/inference/generator.cpp:47-56, EOS ignored).  Weights are
synthetic N(0, 0.02) BF16 from seed 0, prompt ids uniform from seed 1.  With
N > 1 the model is tensor-parallel over N GPUs (strong scaling: the same
model and window, the work split by heads / MLP columns / vocabulary).

Rank 0 prints one JSON line.  The kernel roofline describes the timed path:
after the timed region, a few decode steps of the same CUDA graph are traced
in-graph (q3_engine_trace: per launch and CTA, %globaltimer at start and
end); each launch's share of the traced step times the CUDA-event time per
token of the timed region gives its time per step.  At N = 1 the reference's
own cuBLAS CUDA backend and the reference's Model::forward on this library's
drop-in Backend are timed on the same GPU (bounded samples), and the
reference's CPU backend on the host cores.  `--impl reference` times the
reference's own CPU implementation (its AVX-512 backend compiled from its
sources, oracle/_ref/libref_cpu.so) on bounded samples of the same workload.
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
LAUNCH_KINDS = ("qkv_gemv", "attention", "o_gemv", "gate_up_gemv", "down_gemv")


def parse_args(argv=None):
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
    ap.add_argument("--tune", default="", help="comma list of opt-in prefill variants (q3_engine_set_tuning): "
                    "tp_prefill, fp8_prefill, or all")
    ap.add_argument("--weights", default="bf16", choices=["bf16", "fp8", "nvfp4"],
                    help="fp8: E4M3 GEMV matrices with per-row power-of-two scales; nvfp4: E2M1 with E4M3 scales "
                         "per 16 columns and power-of-two row scales (each the quantized model, not the "
                         "reference's BF16 model; the CUDA graph path)")
    ap.add_argument("--cpu-sample-seconds", type=float, default=10.0,
                    help="CPU legs: time Model::forward calls for about this long (at least 3 calls)")
    ap.add_argument("--reference-cuda-tokens", type=int, default=32,
                    help="time the reference's own cuBLAS CUDA backend (oracle/_ref/libref_cuda.so) for this "
                         "many Model::forward calls at mid-window context (N = 1; 0 = skip); reported as "
                         "reference_cuda")
    ap.add_argument("--drop-in-tokens", type=int, default=32,
                    help="time the reference's own Model::forward on this library's drop-in Backend "
                         "(oracle/_ref/libref_b200.so) for this many calls at mid-window context (N = 1; 0 = "
                         "skip); reported as drop_in")
    ap.add_argument("--timeline-out", default="", help="write the in-graph launch timeline table here")
    ap.add_argument("--probe", default="", choices=["", "gemv", "attention", "gemv8", "decode", "timeline"],
                    help="no benchmark: fixed launches for ncu captures (gemv, attention, gemv8, decode) or the "
                         "per-launch timeline of one decode step (timeline; under torchrun every rank's)")
    ap.add_argument("--position", type=int, default=0, help="--probe decode / timeline: decode position")
    ap.add_argument("--batch", type=int, default=0,
                    help="batched decode instead (q3_batch): this many sequences of the workload's prompt, one step "
                         "= --window tokens of each (default 64); its own JSON line (N = 1)")
    return ap.parse_args(argv)


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
        # every host thread, whatever the launcher set (torchrun sets 1 per rank);
        # read by the OpenMP runtime when the library below is loaded
        os.environ["OMP_NUM_THREADS"] = str(threads)
        from oracle import ModelConfig

        mc = ModelConfig.make(cfg.hidden, cfg.inter, cfg.layers, cfg.q_heads, cfg.kv_heads, 128, cfg.vocab,
                              pos + max_tokens + 1, tied=cfg.tied)
        try:
            from oracle import RefLib

            impl, self.kind = RefLib("cpu"), "reference"
        except (FileNotFoundError, OSError):
            from oracle import Oracle

            impl, self.kind = Oracle(), "port"
        self.pos, self.max_tokens = pos, max_tokens
        self.m = impl.model(mc, seed=0)
        if self.kind == "reference":
            self.m.fill_kv(pos, seed=7)

    def sample(self, seconds, min_tokens=3):
        """Model::forward calls from context pos for about `seconds` (at least min_tokens):
        (tokens, tok/s)."""
        self.m.token_count = self.pos
        tok, n = 1000, 0
        t0 = time.perf_counter()
        while n < self.max_tokens and (n < min_tokens or time.perf_counter() - t0 < seconds):
            tok = self.m.forward(tok)
            n += 1
        return n, n / (time.perf_counter() - t0)

    def close(self):
        self.m.close()


def host_threads():
    """The CPUs this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_token_cap(cfg, seconds):
    # KV capacity for a time-bounded sample: generous for small models, which run fastest
    return max(8, int(seconds * (400 if cfg.hidden <= 1024 else 60 if cfg.hidden <= 2560 else 30)))


def run_reference(a, cfg, prompt_len, capacity, workload):
    """--impl reference: the reference's CPU implementation, rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = host_threads()
    mid = prompt_len + (capacity - prompt_len) // 2
    per_step = max(1.0, a.cpu_sample_seconds / 2)
    cs = CpuSampler(cfg, mid, cpu_token_cap(cfg, per_step), threads)
    kind = cs.kind
    samples = [cs.sample(per_step) for _ in range(a.warmup + a.steps)][a.warmup:]
    cs.close()
    value = statistics.mean(v for _, v in samples)
    n_tok = round(statistics.mean(n for n, _ in samples))
    sample = (f"about {per_step:.0f} s of decode steps (Model::forward; {n_tok} per bench step on average) of "
              f"{cfg.name} at context {mid} (mid-window of {prompt_len}->{capacity}), KV cache prefilled with "
              f"synthetic values")
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


# --------------------------------------------------------------------------- in-graph timeline
def launch_names(layers):
    return [k for _ in range(layers) for k in LAUNCH_KINDS] + ["lm_head"]


def summarize_trace(raw):
    """One traced decode step ([ctas, launches, words] of q3_engine_trace) ->
    per-launch spans (us: this launch's last CTA end minus the previous
    launch's; the first launch, whose CTAs start early beside the previous
    step's lm_head, takes the mean span of the later QKV launches), the
    median per-CTA part times (us) and the SM clock."""
    import numpy as np

    raw = raw.astype(np.float64)
    seen = raw[..., 0] > 0
    t0, t1, c0, c1 = raw[..., 0], raw[..., 1], raw[..., 2], raw[..., 3]
    ghz = float(np.median(((c1 - c0) / np.maximum(t1 - t0, 1))[seen]))
    n = raw.shape[1]
    ends = np.array([t1[seen[:, k], k].max() for k in range(n)])
    spans = np.empty(n)
    spans[1:] = (ends[1:] - ends[:-1]) / 1e3
    layers = (n - 1) // 5
    spans[0] = spans[5:n - 1:5].mean() if layers > 1 else (ends[0] - t0[seen[:, 0], 0].min()) / 1e3
    parts = np.zeros((n, 5))
    for k in range(n):
        v = seen[:, k]
        parts[k] = [np.median(raw[v, k, w]) / ghz / 1e3 for w in (4, 5, 6, 7, 9)]
    return {"spans": spans, "parts": parts, "ghz": ghz}


def trace_table(summ, names, header):
    """Per launch kind: mean span and median parts over layers 1..L-1 (us)."""
    import numpy as np

    lines = [header, f"{'launch':14s} {'span':>7s} {'to_wait':>8s} {'prologue':>9s} {'loop':>7s} {'epilogue':>9s} "
                     f"{'peers':>7s}  (us; parts: CTA medians, SM clock {summ['ghz']:.3f} GHz)"]
    rows = {}
    for k, name in enumerate(names):
        if k < 5 and len(names) > 6:
            continue  # layer 0: its QKV launch starts beside the previous step's lm_head
        rows.setdefault(name, []).append([summ["spans"][k]] + list(summ["parts"][k]))
    for name in list(LAUNCH_KINDS) + ["lm_head"]:
        if name in rows:
            m = np.mean(rows[name], axis=0)
            lines.append(f"{name:14s} {m[0]:7.2f} {m[1]:8.2f} {m[2]:9.2f} {m[3]:7.2f} {m[4]:9.2f} {m[5]:7.2f}")
    return "\n".join(lines)


def traced_steps(eng, pos, n):
    """n decode steps of the CUDA-graph path at `pos`, each traced; their records."""
    eng.trace(True)
    out = []
    for _ in range(n):
        eng.set_position(pos)
        eng.step(1)
        eng.sync()
        out.append(eng.read_trace())
    eng.trace(False)
    return out


def launch_bytes(cfg, world, pos, weights="bf16"):
    """Algorithmic bytes of each launch kind of one decode step on one rank:
    the weights, the input vector and the output vector (GEMVs); K and V of
    positions 0..pos of the rank's kv heads plus q and the output (attention)."""
    H, hd = cfg.hidden, cfg.head_dim
    qd, kd = cfg.q_heads * hd // world, cfg.kv_heads * hd // world
    il, vl = cfg.inter // world, cfg.vocab // world
    wb = {"fp8": 1.0, "nvfp4": 0.5625}.get(weights, 2.0)  # bytes per weight (NVFP4: with its block scales)

    def mat(n, k):
        return int(n * k * wb) + (4 * n if wb < 2 else 0) + 2 * k + 2 * n

    return {"qkv_gemv": mat(qd + 2 * kd, H), "attention": 2 * (pos + 1) * kd * 2 + 2 * qd * 2,
            "o_gemv": mat(H, qd), "gate_up_gemv": mat(2 * il, H), "down_gemv": mat(H, il), "lm_head": mat(vl, H)}


def timeline_roofline(summs, names, cfg, world, pos, weights, ms_per_token, peak, peak_kind, traffic_ratio):
    """The roofline of the dominant kernel (gemv_kernel) and of attention on the
    timed path: each launch's time per step = its share of the traced step x
    the CUDA-event time per token of the timed region."""
    import numpy as np

    spans = np.mean([s["spans"] for s in summs], axis=0)
    scale = ms_per_token * 1000.0 / spans.sum()  # traced us -> timed us
    by = launch_bytes(cfg, world, pos, weights)
    kinds = {}
    for k, name in enumerate(names):
        d = kinds.setdefault(name, {"launches": 0, "us": 0.0, "bytes": 0.0})
        d["launches"] += 1
        d["us"] += spans[k] * scale
        d["bytes"] += by[name]
    per_kind = {}
    for name, d in kinds.items():
        per_kind[name] = {"launches_per_step": d["launches"], "us_per_launch": round(d["us"] / d["launches"], 3),
                          "bytes_per_launch": round(d["bytes"] / d["launches"]),
                          "gbs": round(d["bytes"] / d["us"] / 1e3, 1),
                          "frac": round(d["bytes"] / d["us"] / 1e3 / peak, 4),
                          "share_of_step": round(d["us"] / (ms_per_token * 1000.0), 4)}
    gemv = [n for n in kinds if n != "attention"]
    g_us = sum(kinds[n]["us"] for n in gemv)
    g_bytes = sum(kinds[n]["bytes"] for n in gemv)
    g_launch = sum(kinds[n]["launches"] for n in gemv)
    achieved = g_bytes / g_us / 1e3
    return {
        "kernel": "gemv_kernel (every GEMV launch of a decode step on the timed CUDA-graph path)",
        "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
        "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs (burst copy)",
        "traffic": round(traffic_ratio * g_bytes / g_launch) if traffic_ratio else None,
        "algorithmic_bytes_per_launch": round(g_bytes / g_launch), "launch_us_avg": round(g_us / g_launch, 3),
        "launches_per_step": g_launch, "gemv_us_per_step": round(g_us, 1),
        "step_us": round(ms_per_token * 1000.0, 1), "position": pos,
        "time_source": (f"in-graph launch spans (q3_engine_trace, {len(summs)} traced steps at position {pos}) as "
                        "shares of the step, times the CUDA-event time per token of the timed region"),
        "by_launch_kind": per_kind,
    }


# --------------------------------------------------------------------------- probes (fixed launches for ncu)
def probe_gemv(a):
    """Three decode GEMV launches (Qwen3-8B gate/up: 24576 x 4096, 201 MB), then three
    prefill GEMM launches (512 tokens x 4096 -> 24576), random BF16 operands."""
    import torch

    from inference_b200 import B200Backend

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


def probe_attention(a):
    """Three paged decode-attention launches: Qwen3-8B heads (32 q / 8 kv) at position 4095."""
    import torch

    from inference_b200 import B200Backend

    qh, kvh, pos = 32, 8, a.position or 4095
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


def probe_gemv8(a):
    """The gate/up shape with E4M3 weights (three q3_gemv_e4m3), then the BF16 GEMV;
    prints each launch's CUDA-event time (L2 flushed before each)."""
    import torch

    from inference_b200 import B200Backend

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
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1)
            print(f"{name} {ms * 1000:.1f} us {nbytes / ms / 1e6:.0f} GB/s")
    print("ok")


def _probe_engine(a, cfg, cap, rank=0, world=1, local=0, dist=None):
    import inference_b200 as ib

    e = ib.Engine(cfg, capacity=cap, device=local, tp_rank=rank, tp_size=world)
    e.init_synthetic(0)
    tune = [t for t in a.tune.split(",") if t]
    if tune:
        e.tuning = tune
    if dist is not None:
        _attach(e, dist, a.nccl, rank, world)
    return e


def probe_decode(a):
    """Three decode steps of the CUDA-graph path from --position over a synthetic KV
    cache: the only gemv_kernel / attn_kernel launches of the process."""
    import inference_b200 as ib

    cfg, _, cap = ib.WORKLOADS[a.workload]
    pos = a.position or 520
    e = _probe_engine(a, cfg, cap)
    e.set_tokens(ib.prompt_ids(16, vocab=cfg.vocab))
    e.fill_kv(pos)
    e.set_tokens(ib.prompt_ids(pos + 5, vocab=cfg.vocab))
    e.set_position(pos)
    e.step(3)
    e.sync()
    e.close()
    print("ok")


def probe_timeline(a):
    """The CUDA-graph path's launch timeline of one decode step at --position (under
    torchrun: tensor parallel, every rank's table, printed by rank 0)."""
    import inference_b200 as ib

    cfg, _, cap = ib.WORKLOADS[a.workload]
    pos = a.position or 520
    rank, world, local, dist = _tp_setup()
    e = _probe_engine(a, cfg, cap, rank, world, local, dist)
    e.set_tokens(ib.prompt_ids(16, vocab=cfg.vocab))
    e.fill_kv(pos)
    e.set_tokens(ib.prompt_ids(pos + 16, vocab=cfg.vocab))
    e.set_position(pos)
    e.step(4)
    raws = traced_steps(e, pos, 3)
    _close(e, dist)
    names = launch_names(cfg.layers)
    summ = summarize_trace(raws[-1])
    step_us = summ["spans"].sum()
    text = trace_table(summ, names, f"{a.workload} position {pos} rank {rank}/{world}"
                                    f"{' tuning ' + a.tune if a.tune else ''}: step {step_us:.1f} us")
    if dist is None:
        print(text)
        return 0
    texts = [None] * world
    dist.all_gather_object(texts, text)
    if rank == 0:
        print("\n\n".join(texts))
    dist.barrier()
    dist.destroy_process_group()
    return 0


# --------------------------------------------------------------------------- tensor-parallel plumbing
def _tp_setup():
    """Under torchrun (WORLD_SIZE > 1): (rank, world, local device, torch.distributed)
    with an NCCL process group; (0, 1, LOCAL_RANK, None) otherwise."""
    import datetime

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world == 1:
        return 0, 1, local, None
    import torch.distributed as dist

    rank = int(os.environ["RANK"])
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    return rank, world, local, dist


def _attach(eng, dist, nccl, rank, world):
    import inference_b200 as ib

    if nccl:
        obj = [ib.Engine.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        eng.attach_nccl(obj[0])
    else:
        handles = [None] * world
        dist.all_gather_object(handles, eng.peer_handle())
        dist.barrier()  # every rank's exchange buffer exists and is zeroed before anyone writes
        eng.attach_peers(handles)


def _close(eng, dist):
    """Peers store into and read from each rank's exchange buffer: every rank's stream
    is idle, and every rank has reached this point, before any rank frees its buffer."""
    eng.sync()
    if dist is not None:
        dist.barrier()
    eng.close()


# --------------------------------------------------------------------------- GPU leg
def time_reference_model(kind, cfg, mid, n_tok, what):
    """Model::forward calls of the reference's Qwen3 model at context `mid` (KV
    cache filled with synthetic values), one host round trip per call as the
    reference generator runs: tok/s."""
    import torch

    from oracle import ModelConfig, RefLib

    rl = RefLib(kind)
    mc = ModelConfig.make(cfg.hidden, cfg.inter, cfg.layers, cfg.q_heads, cfg.kv_heads, 128, cfg.vocab,
                          mid + n_tok + 2, tied=cfg.tied)
    rm = rl.model(mc, seed=0)
    try:
        rm.fill_kv(mid, seed=7)
        rm.forward(1000)  # the first call sizes the backend's scratch (the reference's flash-attention scratch)
        rm.token_count = mid
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        tok = 1000
        for _ in range(n_tok):
            tok = rm.forward(tok)
        dt = time.perf_counter() - t0
    finally:
        rm.close()
    return {"value": round(n_tok / dt, 3), "unit": "tok/s",
            "sample": f"{n_tok} Model::forward calls at context {mid}, {what}"}


def run_batch(a, cfg, prompt_len, capacity):
    """Batched decode (q3_batch): a.batch sequences, each prompt_len tokens of its
    own seeded ids; after the prefills and a.warmup windows, a.steps windows of
    a.window steps (one token of every sequence per step) are timed with CUDA
    events on the engine's stream.  Weights are read once per step for all
    sequences; every sequence reads its own KV."""
    import numpy as np
    import torch

    import inference_b200 as ib

    if int(os.environ.get("WORLD_SIZE", "1")) != 1 or a.gpus != 1:
        raise SystemExit("--batch runs on one GPU")
    B = a.batch
    window = a.window or 64
    steps_total = (a.warmup + a.steps) * window
    if a.prompt:
        prompt_len = a.prompt
    max_len = min(capacity, prompt_len + steps_total + 1)
    pages_per_seq = (max_len + 63) // 64
    torch.cuda.set_device(0)
    eng = ib.Engine(cfg, capacity=capacity)
    eng.init_synthetic(0)
    bt = ib.Batch(eng, max_seqs=B, pool_pages=B * pages_per_seq)
    for i in range(B):
        bt.add(ib.prompt_ids(prompt_len, seed=100 + i, vocab=cfg.vocab), max_len=max_len)
    stream = torch.cuda.ExternalStream(eng.stream(), device=torch.device("cuda", 0))
    for _ in range(a.warmup):
        bt.step(window)
    eng.sync()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    p_start = bt.position(0)
    with ClockSampler([0]) as clocks:
        ev0.record(stream)
        bt.step(window * a.steps)
        ev1.record(stream)
        eng.sync()
    ms = ev0.elapsed_time(ev1)
    tokens = B * window * a.steps
    tok_s = tokens / (ms / 1000.0)
    # bytes per step: every weight once, each sequence's KV at its position, averaged
    avg_pos = p_start + (window * a.steps - 1) / 2.0
    step_bytes = cfg.weight_bytes() + B * cfg.kv_bytes_per_position() * (avg_pos + 1)
    peak, peak_kind = measured_peaks()
    gbs = step_bytes * (window * a.steps) / (ms / 1000.0) / 1e9
    line = {
        "metric": f"batched decode tok/s, {B} sequences (q3_batch)", "value": round(tok_s, 3), "unit": "tok/s",
        "n_gpus": 1, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 3),
        "higher_is_better": True, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"{a.workload}-batch{B}", "model": cfg.name, "prompt": prompt_len,
                   "decode_tokens_per_sequence_per_step": window, "sequences": B,
                   "positions": [p_start, p_start + window * a.steps - 1],
                   "decode_path": "batched rows: tcgen05 GEMMs, per-row split-KV attention, one CUDA graph per row count"},
        "per_sequence_tok_s": round(tok_s / B, 3),
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "bytes_per_step": int(step_bytes),
                     "peak_source": f"{peak_kind} hbm_gbs"},
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)
    bt.close()
    eng.close()
    return 0


def main(argv=None):
    a = parse_args(argv)
    from inference_b200.config import WORKLOADS

    if a.workload not in WORKLOADS:
        raise SystemExit(f"unknown workload {a.workload}; choose from {sorted(WORKLOADS)}")
    if a.probe:
        return {"gemv": probe_gemv, "attention": probe_attention, "gemv8": probe_gemv8, "decode": probe_decode,
                "timeline": probe_timeline}[a.probe](a) or 0
    cfg, prompt_len, capacity = WORKLOADS[a.workload]
    if a.batch:
        return run_batch(a, cfg, prompt_len, capacity)
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
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE {world}")
    import numpy as np
    import torch

    rank, world, local, dist = _tp_setup()
    import inference_b200 as ib

    eng = ib.Engine(cfg, capacity=capacity, device=local, tp_rank=rank, tp_size=world, weights=a.weights)
    if a.weights != "bf16":
        workload += "-" + a.weights
    eng.init_synthetic(0)
    tune = [t for t in a.tune.split(",") if t]
    if tune:
        eng.tuning = tune
        if "all" in tune:
            tune = sorted(ib.Engine.TUNE_FLAGS)
    if dist is not None:
        _attach(eng, dist, a.nccl, rank, world)

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
        e2e = {"value": round(a.steps * window / dt, 3), "unit": "tok/s",
               "h2d_bytes_per_step": int(prompt_len * 4 + 4), "d2h_bytes_per_step": int(window * 4),
               "includes": "prompt H2D, prefill of the prompt, decode, token D2H"}

    # ---- prefill (informational: the metric is decode tok/s)
    n_pre = prompt_len - 1
    # every layer's four GEMMs, but the last layer stops after its QKV GEMM
    gemm_flop = 2.0 * n_pre * (cfg.layer_matmul_params() * (cfg.layers - 1) +
                               (cfg.q_heads + 2 * cfg.kv_heads) * cfg.head_dim * cfg.hidden)
    attn_flop = 4.0 * cfg.layers * cfg.q_heads * cfg.head_dim * n_pre * (n_pre + 1) / 2.0
    bf16_peak, bf16_kind = measured_bf16_peak()
    batched = (a.weights == "bf16" or "fp8_prefill" in tune) and (world == 1 or "tp_prefill" in tune)
    prefill = {"tokens": n_pre, "ms": round(pre_t, 3), "tok_s": round(n_pre / (pre_t / 1000.0), 1),
               "path": ("batched: tcgen05 GEMMs (TMEM accumulators, TMA), batched split-KV attention"
                        + ("; row-parallel fp32 partials exchanged between ranks" if world > 1 else "")
                        + ("; packed matrices expanded to their BF16 values first" if a.weights != "bf16" else "")
                        if batched else "per-token decode steps"),
               "tflops": round((gemm_flop + attn_flop) / (pre_t / 1000.0) / 1e12 / world, 1),
               "gemm_tflop": round(gemm_flop / 1e12, 3), "attention_tflop": round(attn_flop / 1e12, 3),
               "peak_tflops": bf16_peak, "frac": round((gemm_flop + attn_flop) / (pre_t / 1000.0) / 1e12 / world /
                                                      bf16_peak, 4),
               "peak_kind": bf16_kind}

    # ---- dominant kernel roofline on the timed path (in-graph timeline at mid-window)
    peak, peak_kind = measured_peaks()
    avg_pos = start_pos + (window - 1) / 2.0
    bytes_tok = cfg.weight_bytes(a.weights) + cfg.kv_bytes_per_position() * (avg_pos + 1)
    mid = start_pos + window // 2
    traffic_ratio = read_traffic_ratio(cfg.name)
    names = launch_names(cfg.layers)
    timeline_text = None
    eng.set_position(mid)
    eng.step(2)
    summs = [summarize_trace(r) for r in traced_steps(eng, mid, 4)]
    roofline = timeline_roofline(summs, names, cfg, world, mid, a.weights, ms / tokens, peak, peak_kind,
                                 traffic_ratio)
    timeline_text = trace_table(summs[-1], names, f"{workload} rank {rank}/{world}, one traced step at "
                                                  f"position {mid}: {summs[-1]['spans'].sum():.1f} us traced, "
                                                  f"{ms / tokens * 1000:.1f} us per token timed")
    launches = len(names) * window * a.steps
    # whole-step roofline: weights + average KV read per token over the window, all ranks
    step_roof = {"bytes_per_token": int(bytes_tok), "achieved_gbs": round(bytes_tok * tok_s / 1e9, 1),
                 "peak_gbs": peak * world, "frac": round(bytes_tok * tok_s / 1e9 / (peak * world), 4)}

    # ---- CPU baseline (rank 0, N = 1 only)
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        threads = host_threads()
        try:
            cs = CpuSampler(cfg, mid, cpu_token_cap(cfg, a.cpu_sample_seconds) + 1, threads)
            cs.sample(0, min_tokens=1)
            n_cpu, v = cs.sample(a.cpu_sample_seconds)
            kind = cs.kind
            cs.close()
            cpu = {"value": round(v, 4), "unit": "tok/s", "cores": threads, "kind": kind,
                   "sample": f"{n_cpu} decode steps (about {a.cpu_sample_seconds:.0f} s) of {cfg.name} at context "
                             f"{mid}, KV prefilled with synthetic values"}
        except Exception as exc:  # report, never fail the GPU number
            cpu = {"value": None, "unit": "tok/s", "cores": threads, "kind": "reference", "sample": f"failed: {exc}"}

    # ---- the reference's own Model::forward on the same GPU (rank 0, N = 1): with its
    # cuBLAS CUDA backend, and with this library's drop-in Backend
    timed_refs = {}
    for key, kind, n_req, what in (("reference_cuda", "cuda", a.reference_cuda_tokens,
                                    "reference cuBLAS CUDA backend built from its sources for sm_100a"),
                                   ("drop_in", "b200", a.drop_in_tokens,
                                    "the reference's Model::forward on this library's drop-in Backend "
                                    "(inference_b200/backend_b200/backend.cpp)")):
        if not (rank == 0 and world == 1 and n_req > 0):
            continue
        try:
            timed_refs[key] = time_reference_model(kind, cfg, mid, n_req, what)
        except Exception as exc:
            timed_refs[key] = {"value": None, "unit": "tok/s", "sample": f"failed: {exc}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(tok_s, 3), "unit": "tok/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 3), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": workload, "model": cfg.name, "prompt": prompt_len, "context": capacity,
                       "decode_tokens_per_step": window, "global_batch": 1,
                       "decode_path": "CUDA graph of fused kernels",
                       "parallelism": f"tp{world}", "weight_format": a.weights, "tuning": tune,
                       "tp_exchange": (None if world == 1 else "NCCL allreduce/allgather" if a.nccl else
                                       "peer-memory stores fused into the o/down/lm_head GEMVs (CUDA IPC, NVLink)"),
                       "weights": "random N(0,0.02) seed 0, ids seed 1",
                       "l2_flush": f"not needed: {cfg.weight_bytes(a.weights) / 1e9:.1f} GB of weights streamed per "
                                   f"token >> 126 MB L2"},
            "clocks": clock, "e2e": e2e, "gpu_launches": int(launches),
            "roofline": roofline, "step_roofline": step_roof, "cpu_baseline": cpu, "prefill": prefill,
        }
        line.update(timed_refs)
        print(json.dumps(line), flush=True)
        if a.timeline_out and timeline_text:
            with open(a.timeline_out, "w") as f:
                f.write(timeline_text + "\n")
    _close(eng, dist)
    if dist:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
