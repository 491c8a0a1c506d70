"""bench.py's reference arm on CPU: the one JSON line the benchmark driver reads (same metric,
unit, config and direction as the GPU arm; cpu_baseline and a zero-copy e2e), silence on ranks
other than 0, and the warm-up floor. The GPU arm itself runs only on a B200."""

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
