"""bench.py's host-side arithmetic and its reference arm, on the CPU.

* the per-launch algorithmic bytes the kernel roofline divides by add up to
  the bytes one decode step streams (every weight format, every model);
* the in-graph timeline reduction: launch spans from a synthetic trace, shares
  of the step that sum to one, achieved bandwidth = bytes / time;
* the clock summary's throttle reasons and loaded-clock median;
* `--impl reference`: one JSON line with the contract's keys from rank 0, no
  work and no output on other ranks.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    sys.path.insert(0, ROOT)
    import bench as b

    return b


@pytest.mark.parametrize("weights", ["bf16", "fp8", "nvfp4"])
@pytest.mark.parametrize("model", ["qwen3-0.6b", "qwen3-4b", "qwen3-8b", "qwen3-32b"])
def test_launch_bytes_add_up_to_the_step(bench, model, weights):
    from inference_b200.config import MODELS

    cfg = MODELS[model]
    pos = 1000
    by = bench.launch_bytes(cfg, 1, pos, weights)
    H, hd = cfg.hidden, cfg.head_dim
    qd, kd, I = cfg.q_heads * hd, cfg.kv_heads * hd, cfg.inter
    # each GEMV launch also reads its input vector and writes its output (BF16)
    io = {"qkv_gemv": 2 * H + 2 * (qd + 2 * kd), "o_gemv": 2 * qd + 2 * H, "gate_up_gemv": 2 * H + 4 * I,
          "down_gemv": 2 * I + 2 * H, "lm_head": 2 * H + 2 * cfg.vocab}
    mats = sum(by[k] - io[k] for k in ("qkv_gemv", "o_gemv", "gate_up_gemv", "down_gemv")) * cfg.layers
    mats += by["lm_head"] - io["lm_head"]
    # weight_bytes adds the norm vectors of every layer, the final norm and one embedding row
    vectors = 2 * (2 * H + 2 * hd) * cfg.layers + 2 * (H + H)
    assert mats == cfg.weight_bytes(weights) - vectors
    # attention: K and V of positions 0..pos of every kv head, plus q in and the output
    assert by["attention"] * cfg.layers == cfg.kv_bytes_per_position() * (pos + 1) + 4 * qd * cfg.layers


def test_launch_bytes_split_over_ranks(bench):
    from inference_b200.config import QWEN3_8B as cfg

    one = bench.launch_bytes(cfg, 1, 100)
    for world in (2, 4, 8):
        part = bench.launch_bytes(cfg, world, 100)
        # the sharded matrices' weights divide exactly; the replicated vectors do not
        for k, io in (("gate_up_gemv", 2 * cfg.hidden), ("lm_head", 2 * cfg.hidden)):
            assert (part[k] - io) * world == pytest.approx(one[k] - io, rel=1e-3)


def _trace(ends_ns, ctas=3, clock_ghz=1.5):
    """A [ctas, launches, 10] record whose launch k ends (latest CTA) at ends_ns[k]."""
    n = len(ends_ns)
    raw = np.zeros((ctas, n, 10), np.uint64)
    for c in range(ctas):
        for k, end in enumerate(ends_ns):
            t1 = end - 100 * c  # CTA 0 is the last to finish
            t0 = t1 - 2000
            raw[c, k, 0], raw[c, k, 1] = t0, t1
            raw[c, k, 2], raw[c, k, 3] = 0, int(2000 * clock_ghz)
            raw[c, k, 4:8] = [300, 600, 900, 1200]
            raw[c, k, 9] = 150
    return raw


def test_summarize_trace_spans(bench):
    layers = 3
    names = bench.launch_names(layers)
    assert len(names) == 5 * layers + 1 and names[-1] == "lm_head"
    rng = np.random.default_rng(0)
    ends = np.cumsum(rng.integers(2_000, 40_000, len(names))) + 10**9
    s = bench.summarize_trace(_trace(ends))
    np.testing.assert_allclose(s["spans"][1:], np.diff(ends) / 1e3)
    # layer 0's QKV launch starts beside the previous step's lm_head: it takes the later QKVs' mean
    assert s["spans"][0] == pytest.approx(np.mean(np.diff(ends)[4:len(names) - 2:5]) / 1e3)
    assert s["ghz"] == pytest.approx(1.5)
    np.testing.assert_allclose(s["parts"][0], np.array([300, 600, 900, 1200, 150]) / 1.5 / 1e3)


def test_timeline_roofline_shares_and_bandwidth(bench):
    from inference_b200.config import QWEN3_0P6B as cfg

    names = bench.launch_names(cfg.layers)
    spans = np.linspace(5.0, 25.0, len(names))
    summ = {"spans": spans, "parts": np.zeros((len(names), 5)), "ghz": 1.9}
    ms_per_token = 0.8
    r = bench.timeline_roofline([summ, summ], names, cfg, 1, 500, "bf16", ms_per_token, 6500.0, "measured", None)
    kinds = r["by_launch_kind"]
    assert sum(k["share_of_step"] for k in kinds.values()) == pytest.approx(1.0, abs=1e-3)
    assert sum(k["launches_per_step"] for k in kinds.values()) == len(names)
    # the traced spans are scaled to the timed step
    assert r["step_us"] == pytest.approx(800.0)
    by = bench.launch_bytes(cfg, 1, 500)
    for name, k in kinds.items():
        assert k["bytes_per_launch"] == by[name]
        assert k["gbs"] == pytest.approx(by[name] / k["us_per_launch"] / 1e3, rel=1e-3)
    gemv = [n for n in kinds if n != "attention"]
    g_bytes = sum(kinds[n]["bytes_per_launch"] * kinds[n]["launches_per_step"] for n in gemv)
    assert r["achieved"] == pytest.approx(g_bytes / r["gemv_us_per_step"] / 1e3, rel=1e-3)
    assert r["frac"] == pytest.approx(r["achieved"] / 6500.0, rel=1e-3)
    assert r["traffic"] is None


def test_clock_summary_reasons_and_loaded_median(bench, tmp_path):
    p = tmp_path / "clocks.csv"
    rows = ["0, 1965, 1965, 800.0, 0x0, Not Active, Not Active, Not Active, Not Active",
            "0, 1890, 1965, 990.0, 0x4, Not Active, Not Active, Not Active, Active",
            "0, 1900, 1965, 995.0, 0x4, Not Active, Not Active, Not Active, Active",
            "0, 345, 1965, 100.0, 0x0, Not Active, Not Active, Not Active, Not Active"]  # idle: not under load
    p.write_text("\n".join(rows) + "\n")
    cs = bench.ClockSampler([0])
    cs.path = str(p)
    s = cs.summary()
    assert s["reasons"] == ["sw_power_cap"]
    assert s["sm_mhz"] == 1900.0 and s["sm_max_mhz"] == 1965.0 and s["samples"] == 4
    assert not p.exists()  # the sample file is removed


def _run_reference(env_extra, timeout=600):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                           "qwen3-0.6b-ctx1024", "--steps", "1", "--warmup", "0", "--cpu-sample-seconds", "2"],
                          cwd=ROOT, env=env, capture_output=True, text=True, timeout=timeout)


def test_reference_arm_prints_the_contract_line():
    # torchrun sets OMP_NUM_THREADS=1 per rank; the reference arm uses every host thread anyway
    r = _run_reference({"RANK": "0", "OMP_NUM_THREADS": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tok/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["n_gpus"] == 1 and d["steps"] == 1
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("reference", "port") and cb["sample"]
    assert cb["cores"] == len(os.sched_getaffinity(0))
    assert d["e2e"] == {"value": d["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    assert d["config"]["workload"] == "qwen3-0.6b-ctx1024"


def test_reference_arm_other_ranks_do_nothing():
    r = _run_reference({"RANK": "1", "WORLD_SIZE": "2"}, timeout=120)
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == ""
