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
    assert line["metric"] == bench.METRIC and line["unit"] == "s/step"
    assert line["config"] == bench.flux_config(1) and "model" not in line["config"]
    assert line["higher_is_better"] is False and line["scaling"] == "strong"
    assert line["n_gpus"] == 1 and line["steps"] == 3 and line["warmup"] == 3
    assert line["value"] > 0 and line["ms_per_step"] > 0
    # the value extrapolates one sample (1 + 1 blocks) to FLUX.1's 19 + 38 blocks
    assert line["value"] > line["ms_per_step"] * 1e-3
    assert line["vs_baseline"] is None
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["cores"] >= 1 and cb["kind"] in ("port", "reference")
    assert cb["unit"] == "s/step" and cb["sample"] and cb["extrapolated"] is True
    e2e = line["e2e"]
    assert e2e == {"value": line["value"], "unit": "s/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


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
    a B200): one JSON line with the contract keys, the CPU baseline requested on rank 0 of a
    one-GPU run, compact extras, a section that raises reported as an error entry instead of losing
    the line, and the long details on stderr."""
    import torch
    real_device = torch.device
    monkeypatch.setattr(torch, "device", lambda *a, **k: real_device("cpu"))
    monkeypatch.setattr(torch.cuda, "set_device", lambda *a, **k: None)
    monkeypatch.setattr(torch.cuda, "empty_cache", lambda: None)

    def fake_headline(args, world, rank, dev, peaks, sampler):
        roof = {"bound": "tensor", "achieved": 2200.0, "peak": 3386.4, "unit": "TOPS", "frac": 2200.0 / 3386.4,
                "traffic": None, "kernels": {"attention_flux": {"achieved": 1000.0}}}
        return {"value": 0.055, "ms_per_step": 55.0, "clocks": {"sm_mhz": 1965.0}, "gpu_launches": 100 * args.steps,
                "e2e": {"value": 0.056, "unit": "s/step", "h2d_bytes_per_step": 10, "d2h_bytes_per_step": 5},
                "roofline": roof, "parity_vs_1gpu": None, "finite": True, "details": {"op_breakdown": []}}

    def failing(*a, **k):
        raise RuntimeError("planted failure")

    monkeypatch.setattr(bench, "bench_flux_headline", fake_headline)
    monkeypatch.setattr(bench, "bench_attention_config2", lambda *a, **k: {
        "tops": 950.0, "kernel_ms": 0.25, "prep_ms": 0.027,
        "roofline": {"achieved": 1040.0, "frac": 0.31, "mixed": {"frac": 0.46}}, "ref_mode": {"tops": 880.0},
        "e2e": {"value": 140.0}})
    monkeypatch.setattr(bench, "bench_gemm", lambda args, dev, peaks, cpu_baseline=True: {
        "gemm": {"ms": 0.042, "roofline": {"achieved": 1840.0, "frac": 0.54}},
        "quantizer": {"ms": 0.02, "roofline": {"achieved": 1900.0, "frac": 0.29}},
        "cublaslt_int_mm": {"ms": 0.031, "tops": 2490.0}, "cpu": cpu_baseline})
    monkeypatch.setattr(bench, "bench_reference_gpu", failing)
    monkeypatch.setattr(bench, "_cpu_flux_baseline", lambda: {"value": 40.0, "unit": "s/step", "cores": 1})
    monkeypatch.setattr(bench, "_host_gib_available", lambda: 1e9)
    monkeypatch.setattr(bench, "bench_flux", lambda *a, **k: {"2048px": {"s_per_step": 0.31, "frac_of_roofline": 0.5,
                                                                         "finite": True}, "sides": list(k["sides"])})
    monkeypatch.setattr(bench, "bench_sdxl", lambda *a, **k: {"s_per_step": 0.059, "cpu": k["cpu_baseline"]})
    monkeypatch.setattr(bench, "ClockSampler", lambda *a, **k: None)
    monkeypatch.setattr(sys, "argv", ["bench.py", "--steps", "5", "--warmup", "3"])
    for var in ("WORLD_SIZE", "RANK", "LOCAL_RANK"):
        monkeypatch.delenv(var, raising=False)
    assert bench.main() == 0
    cap = capsys.readouterr()
    out = [ln for ln in cap.out.splitlines() if ln.strip()]
    assert len(out) == 1
    line = json.loads(out[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "roofline", "clocks", "gpu_launches", "e2e", "cpu_baseline"):
        assert key in line, key
    assert line["n_gpus"] == 1 and line["steps"] == 5 and line["metric"] == bench.METRIC
    assert line["unit"] == "s/step" and line["higher_is_better"] is False and line["scaling"] == "strong"
    assert line["value"] == 0.055 and line["gpu_launches"] == 500
    assert line["cpu_baseline"] == {"value": 40.0, "unit": "s/step", "cores": 1}
    kern = line["roofline"]["kernels"]
    assert kern["attention_config2"]["roofline_frac"] == 0.31 and kern["gemm_config1"]["gemm_ms"] == 0.042
    assert kern["quantizer_config1"]["quantizer_roofline_frac"] == 0.29
    ex = line["extras"]
    assert ex["reference_gpu"] == {"error": "RuntimeError: planted failure"}
    assert ex["flux_2048"]["2048px_s_per_step"] == 0.31 and ex["sdxl_unet"]["s_per_step"] == 0.059
    assert len(out[0]) < 3000                         # the driver keeps about 3 KB of stdout
    assert "bench details: " in cap.err
