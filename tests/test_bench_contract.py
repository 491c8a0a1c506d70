"""bench.py on CPU: the reference arm's one JSON line (same metric, unit, config and direction as
the GPU arm; cpu_baseline and a zero-copy e2e), silence on ranks other than 0, the warm-up floor,
and the GPU arm's line assembly with its GPU sections faked (the sections themselves run only on a
B200)."""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def _run(*args, env_extra=None, timeout=300):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=timeout)


def test_reference_arm_prints_one_contract_line():
    r = _run("--impl", "reference", "--steps", "3", "--warmup", "3")
    assert r.returncode == 0, r.stderr
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == bench.METRIC and line["unit"] == "TOPS"
    assert line["config"] == bench.CONFIG and "model" not in line["config"]
    assert line["higher_is_better"] is True and line["scaling"] == "weak"
    assert line["n_gpus"] == 1 and line["steps"] == 3 and line["warmup"] == 3
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert line["vs_baseline"] is None
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["cores"] >= 1 and cb["kind"] in ("port", "reference")
    assert cb["unit"] == "TOPS" and cb["sample"]
    e2e = line["e2e"]
    assert e2e == {"value": line["value"], "unit": "TOPS", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


def test_reference_arm_silent_on_other_ranks():
    r = _run("--impl", "reference", "--steps", "3", "--warmup", "3", env_extra={"RANK": "1"})
    assert r.returncode == 0, r.stderr
    assert r.stdout.strip() == ""


def test_warmup_floor():
    r = _run("--impl", "reference", "--steps", "3", "--warmup", "2")
    assert r.returncode != 0
    assert "--warmup must be >= 3" in r.stderr


@pytest.mark.parametrize("key", ["bf16_tflops", "hbm_gbs", "source"])
def test_peaks_have_a_source(key):
    assert key in bench._peaks()


def test_main_line_assembles_with_gpu_sections_faked(monkeypatch, capsys):
    """The GPU arm's line assembly, with every GPU section replaced by a fake (the sections run on
    a B200): one JSON line with the contract keys, the CPU baselines requested on rank 0 of a
    one-GPU run, and a section that raises reported as an error entry instead of losing the line."""
    import torch
    real_device = torch.device
    monkeypatch.setattr(torch, "device", lambda *a, **k: real_device("cpu"))
    monkeypatch.setattr(torch.cuda, "set_device", lambda *a, **k: None)
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda: None)

    def fake_attention(args, world, mode, sets, plan, out, sampler=None):
        return {"total_ms": 0.27 * args.steps, "prep_ms": 0.027, "main_ms": 0.246,
                "median_ms": {"prep": 0.027, "main": 0.246, "step": 0.273}, "clocks": {"sm_mhz": 1965.0}}

    def failing(*a, **k):
        raise RuntimeError("planted failure")

    monkeypatch.setattr(bench, "bench_attention", fake_attention)
    monkeypatch.setattr(bench, "bench_gemm", lambda args, dev, peaks, cpu_baseline=True: {"cpu": cpu_baseline})
    monkeypatch.setattr(bench, "bench_e2e", failing)
    monkeypatch.setattr(bench, "_cpu_baseline", lambda: {"value": 0.05, "cores": 1})
    monkeypatch.setattr(bench, "bench_flux", lambda *a, **k: {"cpu": k["cpu_baseline"], "sides": list(k["sides"])})
    monkeypatch.setattr(bench, "bench_sdxl", lambda *a, **k: {"cpu": k["cpu_baseline"]})
    monkeypatch.setattr(bench, "ClockSampler", lambda *a, **k: None)
    monkeypatch.setattr(sys, "argv", ["bench.py", "--steps", "5", "--warmup", "3"])
    for var in ("WORLD_SIZE", "RANK", "LOCAL_RANK"):
        monkeypatch.delenv(var, raising=False)
    assert bench.main() == 0
    out = [ln for ln in capsys.readouterr().out.splitlines() if ln.strip()]
    assert len(out) == 1
    line = json.loads(out[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "roofline", "clocks", "gpu_launches", "e2e", "cpu_baseline"):
        assert key in line, key
    assert line["n_gpus"] == 1 and line["steps"] == 5 and line["metric"] == bench.METRIC
    assert abs(line["value"] - bench.ATTN_OPS * 5 / (0.27 * 5e-3) / 1e12) < 1e-6
    roof = line["roofline"]
    assert roof["frac"] == roof["achieved"] / roof["peak"] and 0 < roof["mixed"]["frac"] < 1
    assert line["e2e"] == {"error": "RuntimeError: planted failure"}
    assert line["w8a8_linear"] == {"cpu": True} and line["sdxl_unet"] == {"cpu": True}
    assert line["flux_dit"] == {"cpu": True, "sides": [1024, 2048]}
