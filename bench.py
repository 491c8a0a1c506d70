#!/usr/bin/env python
"""Benchmark of the B200 INT8 hot path (BASELINE metric: INT8 TOPS of the W8A8 GEMM and the INT8
attention vs the dense INT8 peak; FLUX-DiT s/step at 1024^2 on 1/2/4/8 B200).

Headline workload (and config 5's Ulysses split at N > 1): a FLUX.1-schnell-
architecture DiT (19 double + 38 single blocks, hidden 3072, 24 heads of 128, RoPE 16/56/56) with
seeded random bf16 weights, block linears W8A8 (ConvRot 256) and INT8 attention in the reference's
quant mode, at 1024^2 (512 text + 4096 image tokens), batch 1. One step = one Euler flow-matching
step (one forward, CUDA-graph replayed, plus the latent update); the 4-step schedule repeats, the
latent restarting every 4 steps. At N > 1 the tokens are split over the ranks (Ulysses: an NCCL
all-to-all of q/k/v before and of the output after every attention), so the total work is fixed
("strong" scaling); value = s/step of the slowest rank. At N > 1 rank 0 also runs the same seeded
4-step sample on one GPU and the line reports the N-rank result's distance from it.

The line also carries the dominant kernel's roofline (the W8A8 GEMMs of one forward, timed per
launch with CUDA events) with the other hot kernels beside it (attention in the FLUX step and on
BASELINE config 2, the config-1 W8A8 linear and quantizer), the end-to-end step through the
public API with host copies, clocks, and compact extras (the 2048^2 step, the SDXL UNet step, the
reference's own GPU path timed on this GPU). The full per-section details go to stderr as one JSON
line ("bench details: ..."). Beside the GPU number (rank 0 of a one-GPU run) the reference's CPU
path for the same step runs on this host's cores, extrapolated from one block of each kind.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--only SECTION]

N > 1 runs under torch.distributed.run, one rank per GPU.
"""

from __future__ import annotations

import argparse
import contextlib
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

B, H, S, D = 1, 24, 4608, 128
ATTN_OPS = 4 * B * H * S * S * D                     # QK^T (int8) + PV (bf16), 2 ops per MAC
GEMM_M, GEMM_N, GEMM_K = 4096, 3072, 3072
GEMM_OPS = 2 * GEMM_M * GEMM_N * GEMM_K
ATTN_METRIC = "INT8 TOPS, INT8 flash attention (BASELINE config 2: B=1, H=24, S=4608, D=128, bf16)"
FLUX_SIDE = 1024
METRIC = ("FLUX.1-architecture DiT s/step at 1024^2 (512 text + 4096 image tokens, W8A8 linears, INT8 attention), "
          "Ulysses over the N GPUs")
# DRAM bytes per launch (ncu dram__bytes_read.sum + dram__bytes_write.sum, one capture of each
# kernel on these workloads): attention main kernel (config 2), W8A8 GEMM (config 1), activation
# quantizer (config 1).
TRAFFIC_ATTN = 60.71e6
TRAFFIC_GEMM = 22.09e6
TRAFFIC_QUANT = 25.21e6
ATTN_CONFIG = {"workload": "int8_flash_attention_config2", "batch": B, "heads": H, "seq_len": S, "head_dim": D,
               "quant": "per-64-token-block Q and K (block64)", "causal": False,
               "l2": "4 rotating input sets (4 x 85 MB > 126 MB L2)"}


def _peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        p = json.loads(path.read_text())
        return {"bf16_tflops": float(p["bf16_tflops"]), "hbm_gbs": float(p["hbm_gbs"]), "source": "measured"}
    return {"bf16_tflops": 1590.0, "hbm_gbs": 6650.0, "source": "fallback"}


def _int8_peak_tops(peaks: dict) -> float:
    # B200 dense INT8 runs at twice the dense BF16 rate (4.5 vs 2.25 P nominal).
    return 2.0 * peaks["bf16_tflops"]


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while the GPU is under load."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, out_path: Path | None = None):
        self.gpu_index, self.proc, self.out_path = gpu_index, None, out_path

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu_index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(", ") for r in out.strip().splitlines() if r.count(",") >= 8]
        if self.out_path is not None:
            self.out_path.write_text(out)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows]
        smax = float(rows[0][2])
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.strip() == "Active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": smax, "reasons": reasons, "samples": len(rows),
                "power_w_max": max(float(r[3]) for r in rows)}


def _dist():
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1 and not dist.is_initialized():
        import datetime
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def _guarded(fn, *args, **kwargs) -> dict:
    """fn(*args, **kwargs), or {"error": why} if it raises: a section after the headline that fails
    (out of memory, a missing optional piece) is reported in the line instead of losing it."""
    try:
        return fn(*args, **kwargs)
    except Exception as exc:                         # noqa: BLE001
        import traceback
        traceback.print_exc(file=sys.stderr)
        return {"error": f"{type(exc).__name__}: {exc}"[:300]}


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ─── CPU side: the oracle port of the reference's path ──────────────────────────────────

def _cpu_attention_sample(rows: int, threads: int, mode: str = "block64") -> tuple[float, int]:
    """Seconds for the oracle's int8 attention over ``rows`` query rows of one head against all S
    keys (same shapes / distributions as config 2). Returns (seconds, ops)."""
    import numpy as np
    import oracle
    oracle.set_threads(threads)
    rng = np.random.default_rng(0)
    q = oracle.to_bits(rng.standard_normal((1, rows, 1, D), dtype=np.float32), "bf16")
    k = oracle.to_bits(rng.standard_normal((1, S, 1, D), dtype=np.float32), "bf16")
    v = oracle.to_bits(rng.standard_normal((1, S, 1, D), dtype=np.float32), "bf16")
    t0 = time.perf_counter()
    oracle.attn_int8(q, k, v, "bf16", D ** -0.5, mode)
    return time.perf_counter() - t0, 4 * rows * S * D


def _cpu_baseline(budget_s: float = 15.0) -> dict:
    threads = os.cpu_count() or 1
    rows = 64
    t, ops = _cpu_attention_sample(rows, threads)
    # grow the sample to roughly the time budget (bounded)
    rows = int(max(64, min(S, rows * budget_s / max(t, 1e-3) / 4)) // 64 * 64)
    t, ops = _cpu_attention_sample(rows, threads)
    return {"value": ops / t / 1e12, "unit": "TOPS", "cores": threads, "kind": "port",
            "sample": f"oracle int8 attention (block64), 1 head x {rows} query rows x {S} keys, D={D}, "
                      f"{t:.2f} s", "cpu": _cpu_model(), "reference_sdpa": _cpu_sdpa(threads)}


def _cpu_sdpa(threads: int, reps: int = 2) -> dict:
    """The reference's CPU path for this attention (torch scaled_dot_product_attention in bf16: its
    attention dispatch falls back to it off the GPU) on config 2's full shape, all host cores."""
    import torch
    import torch.nn.functional as F
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        g = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(B, H, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
        F.scaled_dot_product_attention(q, k, v)
        t0 = time.perf_counter()
        for _ in range(reps):
            F.scaled_dot_product_attention(q, k, v)
        sec = (time.perf_counter() - t0) / reps
    finally:
        torch.set_num_threads(prev)
    return {"value": ATTN_OPS / sec / 1e12, "unit": "TOPS", "ms_per_call": sec * 1e3, "cores": threads,
            "sample": f"whole config 2 (B={B}, H={H}, S={S}, D={D}, bf16), {reps} calls after one warm-up"}


def _cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def _cpu_sdpa_heads(heads: int, threads: int) -> float:
    """Seconds for torch's CPU scaled_dot_product_attention over `heads` heads of config 2."""
    import torch
    import torch.nn.functional as F
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(heads)
    q, k, v = (torch.randn(B, heads, S, D, generator=g).to(torch.bfloat16) for _ in range(3))
    t0 = time.perf_counter()
    F.scaled_dot_product_attention(q, k, v)
    return time.perf_counter() - t0


def run_reference(args) -> int:
    """The reference arm: the reference's CPU path for the headline step on this host's cores, rank
    0 only (the other ranks of a torchrun launch exit without work). Off the GPU the reference runs
    its torch-op W8A8 linears (torch._int_mm) and SDPA attention in bf16; `oracle/torch_ref.py`'s
    FluxOps restates those ops and the FLUX runner drives them (pinned bit for bit to the
    reference's own FLUX on the tiny fixture, tests/test_flux_host.py). A whole step takes minutes
    on a CPU, so each timed step is one bounded sample: one forward of the full-width model with one
    double- and one single-stream block at 1024^2, extrapolated to the 19 + 38 blocks of FLUX.1
    (value = 19 x double + 38 x single + the rest of the forward, in s/step); ms_per_step is the
    sample's own wall time."""
    if int(os.environ.get("RANK", "0")) != 0:
        return 0
    step = CpuFluxStep()
    for _ in range(args.warmup):
        step.sample()
    samples = [step.sample() for _ in range(args.steps)]
    value = statistics.mean(x["s_step"] for x in samples)
    wall = statistics.mean(x["wall_s"] for x in samples)
    sample = ("one forward of a full-width FLUX.1 (hidden 3072, 24 heads) with one double- and one single-stream "
              "block at 1024^2 (512 + 4096 tokens) per step, extrapolated to 19 + 38 blocks; torch-op W8A8 "
              "linears (torch._int_mm), SDPA attention, bf16")
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "s/step", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall * 1e3,
            "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16 (torch-op int8 GEMMs)",
            "data": "synthetic: seeded random weights, N(0,1) latent and text", "config": flux_config(args.gpus),
            "cpu_baseline": {"value": value, "unit": "s/step", "cores": step.threads, "kind": "port",
                             "sample": sample, "extrapolated": True, "cpu": _cpu_model(),
                             "s_per_double_block": statistics.mean(x["double"] for x in samples),
                             "s_per_single_block": statistics.mean(x["single"] for x in samples),
                             "s_rest_of_forward": statistics.mean(x["rest"] for x in samples)},
            "e2e": {"value": value, "unit": "s/step", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ─── GPU side ───────────────────────────────────────────────────────────────────────────

def _events(n):
    import torch
    return [torch.cuda.Event(enable_timing=True) for _ in range(n)]


def _cpu_runahead() -> None:
    """Queue ~50 ms of GPU sleep before a timed region so the host enqueues the timed launches
    ahead of the GPU: the CUDA events then time kernels back to back, not host launch latency."""
    import torch
    torch.cuda._sleep(100_000_000)


def bench_attention(args, world, mode_code, sets, plan, out, sampler=None):
    """Times K steps of prep + main over rotating input sets. Returns dict of timings (ms)."""
    import torch
    scale = D ** -0.5
    for i in range(args.warmup):
        q, k, v = sets[i % len(sets)]
        plan(q, k, v, out, scale)
    torch.cuda.synchronize()
    if sampler is not None:
        # clock soak: the same step for ~1 s right before the timed region, sampled with it
        sampler.start()
        t_end = time.perf_counter() + 1.0
        i = 0
        while time.perf_counter() < t_end:
            q, k, v = sets[i % len(sets)]
            plan(q, k, v, out, scale)
            i += 1
            if i % 50 == 0:
                torch.cuda.synchronize()
        torch.cuda.synchronize()
    ev = _events(3 * args.steps)
    start, end = _events(2)
    _barrier(world)
    torch.cuda.synchronize()
    _cpu_runahead()
    start.record()
    for i in range(args.steps):
        q, k, v = sets[i % len(sets)]
        ev[3 * i].record()
        plan.prep(q, k)
        ev[3 * i + 1].record()
        plan.main(v, out, scale)
        ev[3 * i + 2].record()
    end.record()
    torch.cuda.synchronize()
    _barrier(world)
    clocks = sampler.stop() if sampler is not None else None
    total = start.elapsed_time(end)
    preps = [ev[3 * i].elapsed_time(ev[3 * i + 1]) for i in range(args.steps)]
    mains = [ev[3 * i + 1].elapsed_time(ev[3 * i + 2]) for i in range(args.steps)]
    return {"total_ms": total, "prep_ms": sum(preps) / args.steps, "main_ms": sum(mains) / args.steps,
            "median_ms": {"prep": statistics.median(preps), "main": statistics.median(mains),
                          "step": statistics.median(a + b for a, b in zip(preps, mains))},
            "clocks": clocks}


def _e2e_serial(args, dev):
    """bench_e2e without overlap: copy-in, compute and copy-out of each step on one stream."""
    import torch
    from diffucore_b200 import _attention
    g = torch.Generator().manual_seed(1)
    host = [torch.randn(B, H, S, D, generator=g).to(torch.bfloat16).pin_memory() for _ in range(3)]
    host_out = torch.empty(B, S, H * D, dtype=torch.bfloat16).pin_memory()

    def step():
        q, k, v = (t.to(dev, non_blocking=True) for t in host)
        o = _attention.attention_bhld(q, k, v, "int8_turing", quant_mode="block64")
        host_out.copy_(o, non_blocking=True)

    for _ in range(max(3, args.warmup // 4)):
        step()
    torch.cuda.synchronize()
    n = max(3, min(args.steps, 50))
    s, e = _events(2)
    s.record()
    for _ in range(n):
        step()
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / n
    return {"value": ATTN_OPS / (ms * 1e-3) / 1e12, "unit": "TOPS", "ms_per_step": ms,
            "h2d_bytes_per_step": 3 * B * H * S * D * 2, "d2h_bytes_per_step": B * S * H * D * 2, "steps": n,
            "pipelined": False}


def bench_e2e(args, dev):
    """bench_e2e_pipelined, or the serial form (with the reason) if that one raises."""
    try:
        return bench_e2e_pipelined(args, dev)
    except Exception as exc:                      # keep the bench line; say why it is the serial form
        out = _e2e_serial(args, dev)
        out["pipelined_error"] = f"{type(exc).__name__}: {exc}"[:200]
        return out


def bench_e2e_pipelined(args, dev):
    """The same metric through the public API (attention_bhld) with pinned host inputs copied in
    and the output copied back inside the timed region, every step.

    Steps are pipelined the way a serving loop runs them: step i+1's inputs are copied in on one
    stream (into the other of two device input sets) while step i computes on a second and step
    i-1's output is copied out on a third, so the steady state is bound by the slowest of the
    host-to-device copy, the kernels and the device-to-host copy rather than their sum. The last
    step's output is compared with a serial run of the same call."""
    import torch
    from diffucore_b200 import _attention
    g = torch.Generator().manual_seed(1)
    host = [torch.randn(B, H, S, D, generator=g).to(torch.bfloat16).pin_memory() for _ in range(3)]
    host_out = torch.empty(B, S, H * D, dtype=torch.bfloat16).pin_memory()
    dev_in = [[torch.empty(B, H, S, D, dtype=torch.bfloat16, device=dev) for _ in range(3)] for _ in range(2)]
    s_in, s_comp, s_out = (torch.cuda.Stream(device=dev) for _ in range(3))
    comp_done = [None, None]

    def step(i):
        b = i % 2
        with torch.cuda.stream(s_in):
            if comp_done[b] is not None:
                s_in.wait_event(comp_done[b])          # step i-2 has finished reading this set
            for d_t, h_t in zip(dev_in[b], host):
                d_t.copy_(h_t, non_blocking=True)
            in_done = torch.cuda.Event()
            in_done.record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(in_done)
            o = _attention.attention_bhld(*dev_in[b], "int8_turing", quant_mode="block64")
            done = torch.cuda.Event()
            done.record(s_comp)
            comp_done[b] = done
        with torch.cuda.stream(s_out):
            s_out.wait_event(done)
            host_out.copy_(o, non_blocking=True)
            o.record_stream(s_out)                   # o is freed only after its copy-out

    def run(first, count):
        cur = torch.cuda.current_stream(dev)
        start, end = _events(2)
        start.record(cur)
        for st in (s_in, s_comp, s_out):
            st.wait_stream(cur)
        for i in range(first, first + count):
            step(i)
        for st in (s_in, s_comp, s_out):
            cur.wait_stream(st)
        end.record(cur)
        return start, end

    run(0, max(3, args.warmup // 4))
    torch.cuda.synchronize()
    n = max(3, min(args.steps, 50))
    start, end = run(0, n)
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / n
    ref = _attention.attention_bhld(*(t.to(dev) for t in host), "int8_turing", quant_mode="block64").cpu()
    return {"value": ATTN_OPS / (ms * 1e-3) / 1e12, "unit": "TOPS", "ms_per_step": ms,
            "h2d_bytes_per_step": 3 * B * H * S * D * 2, "d2h_bytes_per_step": B * S * H * D * 2, "steps": n,
            "pipelined": "copy-in, compute and copy-out on three streams, two device input sets",
            "output_matches_serial_call": bool(torch.equal(host_out, ref))}


def bench_gemm(args, dev, peaks, cpu_baseline: bool = True):
    """Config 1: W8A8 linear (quantize + tcgen05 GEMM with rescale/bias epilogue). With
    `cpu_baseline` (rank 0 of a one-GPU run only) the reference's CPU path is timed beside it."""
    import torch
    from diffucore_b200 import _int8, kernels
    g = torch.Generator().manual_seed(0)
    lin = torch.nn.Linear(GEMM_K, GEMM_N, bias=True).to(torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_((torch.randn(GEMM_N, GEMM_K, generator=g) * 0.02).to(torch.bfloat16))
        lin.bias.copy_((torch.randn(GEMM_N, generator=g) * 0.01).to(torch.bfloat16))
    layer = _int8.Int8Linear.from_linear(lin.to(dev), group=0)
    nsets = 6                                               # 6 x (25 MB x + 13 MB q + 25 MB y) > L2
    xs = [torch.randn(GEMM_M, GEMM_K, generator=g).to(torch.bfloat16).to(dev) for _ in range(nsets)]
    qs = [kernels.quant_rows(x, 0) for x in xs]
    steps = max(10, args.steps)
    for i in range(max(3, args.warmup)):
        q, s = qs[i % nsets]
        layer.matmul_quantized(q, s, torch.bfloat16)
        kernels.quant_rows(xs[i % nsets], 0)
    torch.cuda.synchronize()
    ev = _events(3 * steps)
    _cpu_runahead()
    for i in range(steps):
        x = xs[i % nsets]
        ev[3 * i].record()
        q, s = kernels.quant_rows(x, 0)
        ev[3 * i + 1].record()
        layer.matmul_quantized(q, s, torch.bfloat16)
        ev[3 * i + 2].record()
    torch.cuda.synchronize()
    quants = [ev[3 * i].elapsed_time(ev[3 * i + 1]) for i in range(steps)]
    gemms = [ev[3 * i + 1].elapsed_time(ev[3 * i + 2]) for i in range(steps)]
    quant_ms, gemm_ms = sum(quants) / steps, sum(gemms) / steps
    # the library GEMM bar: cuBLASLt int8 GEMM (torch._int_mm, the reference's GEMM on this GPU)
    ev2 = _events(2)
    qa = [q for q, _ in qs]
    wt = layer.weight.t()
    for i in range(3):
        torch._int_mm(qa[i % nsets], wt)
    torch.cuda.synchronize()
    _cpu_runahead()
    ev2[0].record()
    for i in range(steps):
        torch._int_mm(qa[i % nsets], wt)
    ev2[1].record()
    torch.cuda.synchronize()
    cublas_ms = ev2[0].elapsed_time(ev2[1]) / steps
    tops = GEMM_OPS / (gemm_ms * 1e-3) / 1e12
    peak = _int8_peak_tops(peaks)
    qbytes = GEMM_M * GEMM_K * 2 + GEMM_M * GEMM_K + GEMM_M * 4
    qgbs = qbytes / (quant_ms * 1e-3) / 1e9
    return {
        "workload": "W8A8 linear, BASELINE config 1: M=4096, K=N=3072, bf16 in/out, bias, group 0",
        "value": GEMM_OPS / ((quant_ms + gemm_ms) * 1e-3) / 1e12, "unit": "TOPS",
        "ms_per_call": quant_ms + gemm_ms,
        "median_ms": {"quantizer": statistics.median(quants), "gemm": statistics.median(gemms)},
        "gemm": {"ms": gemm_ms, "roofline": {"bound": "tensor", "achieved": tops, "peak": peak, "unit": "TOPS",
                                             "frac": tops / peak, "traffic": TRAFFIC_GEMM,
                                             "peak_source": f"2 x bf16_tflops ({peaks['source']})"}},
        "quantizer": {"ms": quant_ms, "roofline": {"bound": "hbm", "achieved": qgbs, "peak": peaks["hbm_gbs"],
                                                   "unit": "GB/s", "frac": qgbs / peaks["hbm_gbs"],
                                                   "traffic": TRAFFIC_QUANT, "peak_source": f"hbm_gbs ({peaks['source']})"}},
        "gpu_launches_per_call": 2,
        "cublaslt_int_mm": {"ms": cublas_ms, "tops": GEMM_OPS / (cublas_ms * 1e-3) / 1e12,
                            "note": "torch._int_mm (cuBLASLt), int32 out, no quantize/rescale: the "
                                    "reference's GEMM on this GPU"},
        **({"cpu_baseline": _cpu_linear_baseline()} if cpu_baseline else {}),
    }


def _cpu_linear_baseline(reps: int = 3) -> dict:
    """Config 1 through the reference's CPU path (its torch-op Int8Linear forward, restated in
    oracle/torch_ref.py and pinned to its output hashes) on all host cores, whole workload."""
    import torch
    from oracle import torch_ref
    threads = os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        g = torch.Generator().manual_seed(0)
        x = torch.randn(GEMM_M, GEMM_K, generator=g).to(torch.bfloat16)
        w = (torch.randn(GEMM_N, GEMM_K, generator=g) * 0.02).to(torch.bfloat16)
        b = (torch.randn(GEMM_N, generator=g) * 0.01).to(torch.bfloat16)
        wq, ws = torch_ref.quantize_weight(w, 0)
        torch_ref.int8_linear(x, wq, ws, b, 0)                       # warm-up
        t0 = time.perf_counter()
        for _ in range(reps):
            torch_ref.int8_linear(x, wq, ws, b, 0)
        sec = (time.perf_counter() - t0) / reps
    finally:
        torch.set_num_threads(prev)
    return {"value": GEMM_OPS / sec / 1e12, "unit": "TOPS", "ms_per_call": sec * 1e3, "cores": threads,
            "kind": "port", "sample": f"whole config 1 (M={GEMM_M}, K=N={GEMM_K}), {reps} calls after one warm-up",
            "note": "the reference's torch-op Int8Linear forward (quantize rows, torch._int_mm, rescale)",
            "cpu": _cpu_model()}


# ─── FLUX-architecture DiT (BASELINE configs 4 and 5) ────────────────────────────────────

FLUX_STEPS = 4          # Euler flow-matching steps (FLUX.1 [schnell], shift 1)
FLUX_TXT = 512


def flux_work(L: int, C: int = 3072, F: int = 12288, H: int = 24, Dh: int = 128, blocks: int = 57) -> dict:
    """Algorithmic work of one FLUX.1 forward over L tokens: every block's token-wise linears are
    24 L C^2 int8 ops (double: qkv 6, proj 2, MLP 16 per stream row; single: linear1 14, linear2 10),
    its attention 2 L^2 Dh H int8 ops (QK^T) + 2 L^2 Dh H bf16 ops (PV)."""
    lin = blocks * 24 * L * C * C
    att = blocks * 2 * L * L * Dh * H
    return {"linear_int8_ops": lin, "attn_int8_ops": att, "attn_bf16_ops": att}


def _host_gib_available() -> float:
    """Host memory this process can still use, GiB: the system's available memory, capped by a
    cgroup (v2) limit when one is set."""
    try:
        import psutil
        avail = psutil.virtual_memory().available
    except Exception:                                    # noqa: BLE001  no psutil: assume enough
        return float("inf")
    try:
        limit = Path("/sys/fs/cgroup/memory.max").read_text().strip()
        used = int(Path("/sys/fs/cgroup/memory.current").read_text().strip())
        if limit != "max":
            avail = min(avail, int(limit) - used)
    except (OSError, ValueError):
        pass
    return avail / 2 ** 30


HOST_GIB_FOR_CPU_BASELINES = 16.0      # measured peaks: ~6 GiB (SDXL in fp32), ~3 GiB (FLUX blocks)


class CpuFluxStep:
    """The reference's CPU path for one FLUX.1 step at 1024^2 on all host cores, extrapolated from
    one block of each kind (a whole step takes minutes on a CPU): a full-width model (hidden 3072,
    24 heads, RoPE 16/56/56) with one double- and one single-stream block, random bf16 weights,
    block linears W8A8 with ConvRot 256, 512 text + 4096 image tokens, run by the FLUX runner with
    the reference's torch ops (oracle/torch_ref.py FluxOps: torch._int_mm W8A8 linears, SDPA
    attention; pinned to the reference's own FLUX output in tests/test_flux_host.py). One
    :meth:`sample` = one forward of that model; step = 19 x double block + 38 x single block + the
    rest of the forward (embedders, modulations, final layer)."""

    def __init__(self, threads: int | None = None):
        import torch
        from diffucore_b200 import _lib, flux
        from oracle.torch_ref import FluxOps
        self.threads = threads or os.cpu_count() or 1
        prev = torch.get_num_threads()
        torch.set_num_threads(self.threads)
        try:
            t0 = time.perf_counter()
            model = flux.build_flux(flux.FluxConfig(depth=1, depth_single_blocks=1), seed=0, device="cpu", group=256)
            self.build_s = time.perf_counter() - t0
            lat = FLUX_SIDE // 8
            n_img = (lat // 2) ** 2
            self.runner = flux.FluxRunner(model, FLUX_TXT, n_img, device="cpu", attn_mode=_lib.MODE_REF, ops=FluxOps())
            self.runner.set_positions(flux.img_ids(lat, lat, 2), flux.txt_ids(FLUX_TXT))
            g = torch.Generator().manual_seed(1)
            self.x = flux.patchify(torch.randn(1, 16, lat, lat, generator=g)).to(torch.bfloat16)[0]
            self.txt = torch.randn(FLUX_TXT, 4096, generator=g).to(torch.bfloat16)
            self.y = torch.randn(1, 768, generator=g).to(torch.bfloat16)
            self.ts = torch.full((1,), 1.0, dtype=torch.bfloat16)
        finally:
            torch.set_num_threads(prev)
        self.secs = {"double": 0.0, "single": 0.0}

        def timed(fn, key):
            def wrapper(*a, **k):
                t = time.perf_counter()
                r = fn(*a, **k)
                self.secs[key] += time.perf_counter() - t
                return r
            return wrapper

        self.runner._double = timed(self.runner._double, "double")
        self.runner._single = timed(self.runner._single, "single")

    def sample(self) -> dict:
        import torch
        prev = torch.get_num_threads()
        torch.set_num_threads(self.threads)
        try:
            self.secs.update(double=0.0, single=0.0)
            t0 = time.perf_counter()
            v = self.runner.forward(self.x, self.txt, self.ts, self.y)
            total = time.perf_counter() - t0
        finally:
            torch.set_num_threads(prev)
        rest = total - self.secs["double"] - self.secs["single"]
        return {"s_step": 19 * self.secs["double"] + 38 * self.secs["single"] + rest, "wall_s": total,
                "double": self.secs["double"], "single": self.secs["single"], "rest": rest,
                "finite": bool(torch.isfinite(v).all())}


def _cpu_flux_baseline() -> dict:
    """:class:`CpuFluxStep` after one warm-up forward, one measured forward (rank 0 of a one-GPU run)."""
    step = CpuFluxStep()
    step.sample()
    r = step.sample()
    return {"value": r["s_step"], "unit": "s/step", "cores": step.threads, "kind": "port", "extrapolated": True,
            "s_per_double_block": r["double"], "s_per_single_block": r["single"], "s_rest_of_forward": r["rest"],
            "sample": "1 double + 1 single full-width block at 1024^2, measured; step = 19 x double + "
                      "38 x single + rest (torch-op int8 linears, SDPA, bf16)",
            "finite": r["finite"]}


def bench_flux(args, world, rank, dev, peaks, sides=(1024, 2048), cpu_baseline: bool = False) -> dict:
    """Seconds per Euler step of the FLUX.1-architecture DiT (random bf16 weights, block linears
    W8A8 with ConvRot group 256, INT8 attention in the reference's quant mode) at the given image
    sides: 1024 -> 512 text + 4096 image tokens, 2048 -> 512 + 16384. With world > 1 the tokens are
    split over the ranks (Ulysses all-to-all around every attention). With `cpu_baseline` (rank 0
    of a one-GPU run) the 1024^2 entry also carries the reference's CPU path, extrapolated."""
    import torch
    import torch.distributed as dist
    from diffucore_b200 import _attention, _lib, flux
    t0 = time.perf_counter()
    model = flux.build_flux(flux.FluxConfig(), seed=0, device=dev, group=256)
    _attention.set_attention_backend(model, "int8_turing")
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    pg = dist.group.WORLD if world > 1 else None
    int8_peak = _int8_peak_tops(peaks) * 1e12
    bf16_peak = peaks["bf16_tflops"] * 1e12
    out = {"model": "FLUX.1-schnell architecture (19 double + 38 single blocks, 3072 hidden, 24 heads), "
                    "random bf16 weights, block linears W8A8 (ConvRot 256), INT8 attention (mode ref)",
           "steps": FLUX_STEPS, "sampler": "euler, shift 1", "build_s": build_s}
    for side in sides:
        lat = side // 8
        n_img = (lat // 2) ** 2
        L = FLUX_TXT + n_img
        runner = flux.FluxRunner(model, FLUX_TXT, n_img, process_group=pg, device=dev, attn_mode=_lib.MODE_REF)
        runner.set_positions(flux.img_ids(lat, lat, 2, device=dev), flux.txt_ids(FLUX_TXT, device=dev))
        g = torch.Generator(device=dev).manual_seed(1)
        x_all = flux.patchify(torch.randn(1, 16, lat, lat, generator=g, device=dev)).to(torch.bfloat16)[0]
        txt_all = torch.randn(FLUX_TXT, 4096, generator=g, device=dev).to(torch.bfloat16)
        y = torch.randn(1, 768, generator=g, device=dev).to(torch.bfloat16)
        i0, i1 = runner.img_rows
        r0 = runner.rows[0]
        x, txt = x_all[i0:i1].contiguous(), txt_all[r0: r0 + runner.t_loc].contiguous()
        sigmas = flux.flow_schedule(FLUX_STEPS, 1.0)
        res = {}
        for mode in ("eager", "graph"):
            step_fn = runner
            if mode == "graph":
                try:
                    step_fn = flux.FluxGraph(runner, x, txt, y)
                except Exception as exc:                    # report, keep the eager number
                    res["graph_error"] = f"{type(exc).__name__}: {exc}"[:300]
                    break
            xo = flux.euler_sample(step_fn, x, txt, y, sigmas)       # warm-up: one whole sampling run
            torch.cuda.synchronize()
            _barrier(world)
            s, e = _events(2)
            s.record()
            xo = flux.euler_sample(step_fn, x, txt, y, sigmas)
            e.record()
            torch.cuda.synchronize()
            res[mode] = _max_over_ranks(s.elapsed_time(e) * 1e-3 / FLUX_STEPS, world)
            res["finite"] = bool(torch.isfinite(xo).all())
            del step_fn
        finite = res.pop("finite")
        s_step = min(v for k, v in res.items() if k in ("eager", "graph"))
        w = flux_work(L)
        compute_s = (w["linear_int8_ops"] + w["attn_int8_ops"]) / int8_peak + w["attn_bf16_ops"] / bf16_peak
        roof = compute_s / world
        a2a = 0.0
        if world > 1:
            Lr = L // world
            per_block = (Lr * 3 * 3072 + Lr * 3072) * 2 * (world - 1) / world      # bytes sent per rank
            a2a = 57 * per_block / 770e9                                          # measured peer copy GB/s
            roof = max(roof, a2a)
        out[f"{side}px"] = {"tokens": L, "s_per_step": s_step, "n_gpus": world,
                            "s_per_step_eager": res.get("eager"), "s_per_step_graph": res.get("graph"),
                            **({"graph_error": res["graph_error"]} if "graph_error" in res else {}),
                            "roofline_s_per_step": roof, "frac_of_roofline": roof / s_step,
                            "a2a_s_per_step_at_770GBps": a2a, "finite": finite,
                            "work_per_step": {k: v / 1e12 for k, v in w.items()}, "work_unit": "T ops"}
        del runner, x_all, txt_all, xo
        torch.cuda.empty_cache()
    del model
    torch.cuda.empty_cache()
    if cpu_baseline and "1024px" in out and _host_gib_available() < HOST_GIB_FOR_CPU_BASELINES:
        out["1024px"]["cpu_baseline_error"] = f"skipped: under {HOST_GIB_FOR_CPU_BASELINES:.0f} GiB of host memory free"
    elif cpu_baseline and "1024px" in out:
        try:
            out["1024px"]["cpu_baseline"] = _cpu_flux_baseline()
        except Exception as exc:                    # keep the GPU numbers; say why it is missing
            out["1024px"]["cpu_baseline_error"] = f"{type(exc).__name__}: {exc}"[:300]
    return out


def bench_sdxl(args, dev, peaks, steps: int = 25, cpu_baseline: bool = False) -> dict:
    """SDXL-architecture UNet, random fp16 weights, attention / FF linears W8A8,
    INT8 self-attention (head dim 64), CFG batch 2 at 1024^2 (latent 4 x 128 x 128, context
    [2, 77, 2048], adm [2, 2816]); Euler, 25 steps. s/step = CUDA-event time of a whole 25-step run
    / 25 after a 3-step warm-up; int8 work per step counted by hooks on one forward. With
    `cpu_baseline` (rank 0 of a one-GPU run) the reference's CPU path for one step sits beside it."""
    import torch
    from diffucore_b200 import _int8, unet
    t0 = time.perf_counter()
    model = unet.build_sdxl_unet(seed=0, device=dev)
    build_s = time.perf_counter() - t0
    g = torch.Generator(device=dev).manual_seed(1)
    x = torch.randn(1, 4, 128, 128, generator=g, device=dev).half()
    ctx = torch.randn(2, 77, 2048, generator=g, device=dev).half()
    y = torch.randn(2, 2816, generator=g, device=dev).half()
    work = {"linear_int8_ops": 0, "attn_int8_ops": 0, "attn_f16_ops": 0}
    hooks = []

    def lin_hook(mod, inp, out):
        m = inp[0].numel() // inp[0].shape[-1]
        work["linear_int8_ops"] += 2 * m * mod.in_features * mod.out_features

    def attn_hook(mod, inp, out):
        b, l, _ = inp[0].shape
        if mod.is_selfattn and isinstance(mod.to_q, _int8.Int8Linear):
            # the shared-quantization path calls the three projections' GEMMs directly
            for lin in (mod.to_q, mod.to_k, mod.to_v):
                work["linear_int8_ops"] += 2 * b * l * lin.in_features * lin.out_features
        if mod.attn_backend == "int8_turing":
            ops = 2 * b * mod.heads * l * l * mod.dim_head
            work["attn_int8_ops"] += ops
            work["attn_f16_ops"] += ops
    for m in model.modules():
        if isinstance(m, _int8.Int8Linear):
            hooks.append(m.register_forward_hook(lin_hook))
        elif isinstance(m, unet.CrossAttention):
            hooks.append(m.register_forward_hook(attn_hook))
    with torch.no_grad():
        model(x.expand(2, -1, -1, -1), torch.full((2,), 500.0, device=dev), ctx, y)
    for h in hooks:
        h.remove()
    unet.euler_cfg_sample(model, x, ctx, y, steps=3)
    torch.cuda.synchronize()
    s, e = _events(2)
    s.record()
    out = unet.euler_cfg_sample(model, x, ctx, y, steps=steps)
    e.record()
    torch.cuda.synchronize()
    s_step = s.elapsed_time(e) * 1e-3 / steps
    res = {"model": "SDXL-architecture UNet (320/640/1280, depth 0/2/10, head dim 64, context 2048), random fp16 "
                    "weights, attention / FF linears W8A8 (group 0), INT8 self-attention",
           "batch": "CFG 2", "latent": [4, 128, 128], "sampler": "euler", "steps": steps, "build_s": build_s,
           "s_per_step": s_step, "finite": bool(torch.isfinite(out).all()),
           "int8_work_per_step_T": {k: v / 1e12 for k, v in work.items()}}
    if cpu_baseline and _host_gib_available() < HOST_GIB_FOR_CPU_BASELINES:
        res["cpu_baseline_error"] = f"skipped: under {HOST_GIB_FOR_CPU_BASELINES:.0f} GiB of host memory free"
    elif cpu_baseline:
        del out
        try:
            res["cpu_baseline"] = _cpu_sdxl_baseline(model, x, ctx, y)
        except Exception as exc:                    # keep the GPU numbers; say why it is missing
            res["cpu_baseline_error"] = f"{type(exc).__name__}: {exc}"[:300]
    del model
    torch.cuda.empty_cache()
    return res


def _cpu_sdxl_baseline(model, x, ctx, y) -> dict:
    """The reference's CPU path for one Euler step of config 3 on all host cores: the same UNet
    (the benchmark's own quantized weights) moved to the host in fp32, the reference's compute
    dtype off the GPU, every W8A8 linear through the reference's torch-op forward
    (oracle/torch_ref.py CpuInt8Linear: torch._int_mm) and self-attention through SDPA (the
    attention dispatch's CPU path); one CFG-2 forward is one step's UNet work."""
    import torch
    from oracle.torch_ref import cpu_int8_linears_
    threads = os.cpu_count() or 1
    prev = torch.get_num_threads()
    torch.set_num_threads(threads)
    try:
        model = model.to("cpu", torch.float32)
        n = cpu_int8_linears_(model)
        xc, cc, yc = (t.to("cpu", torch.float32) for t in (x, ctx, y))
        with torch.no_grad():
            t0 = time.perf_counter()
            eps = model(xc.expand(2, -1, -1, -1), torch.full((2,), 500.0), cc, yc)
            sec = time.perf_counter() - t0
    finally:
        torch.set_num_threads(prev)
    return {"value": sec, "unit": "s/step", "cores": threads, "kind": "port",
            "sample": f"one CFG-2 UNet forward (one Euler step's model work) at 1024^2, fp32, {n} W8A8 linears",
            "note": "the reference's CPU path: torch-op W8A8 linears (torch._int_mm), SDPA attention",
            "finite": bool(torch.isfinite(eps).all()), "cpu": _cpu_model()}


def flux_op_breakdown(dev, side: int = 1024) -> dict:
    """GPU time per op kind of one FLUX forward at ``side``^2 on one GPU (after two warm-ups)."""
    import torch
    from diffucore_b200 import _attention, _lib, flux
    model = flux.build_flux(flux.FluxConfig(), seed=0, device=dev, group=256)
    _attention.set_attention_backend(model, "int8_turing")
    lat = side // 8
    n_img = (lat // 2) ** 2
    ops = flux.TimedOps()
    runner = flux.FluxRunner(model, FLUX_TXT, n_img, device=dev, attn_mode=_lib.MODE_REF, ops=ops)
    runner.set_positions(flux.img_ids(lat, lat, 2, device=dev), flux.txt_ids(FLUX_TXT, device=dev))
    g = torch.Generator(device=dev).manual_seed(1)
    x = flux.patchify(torch.randn(1, 16, lat, lat, generator=g, device=dev)).to(torch.bfloat16)[0]
    txt = torch.randn(FLUX_TXT, 4096, generator=g, device=dev).to(torch.bfloat16)
    y = torch.randn(1, 768, generator=g, device=dev).to(torch.bfloat16)
    t = torch.full((1,), 0.5, device=dev, dtype=torch.bfloat16)
    for _ in range(2):
        runner.forward(x, txt, t, y)
    torch.cuda.synchronize()
    ops.events.clear()
    s, e = _events(2)
    s.record()
    runner.forward(x, txt, t, y)
    e.record()
    rows = ops.summary()
    total = s.elapsed_time(e)
    return {"workload": f"FLUX.1 forward, {side}^2 ({FLUX_TXT + n_img} tokens), 1 GPU, eager with events",
            "forward_ms": round(total, 3), "ops_ms": round(sum(r["ms"] for r in rows), 3),
            "other_ms_torch_ops": round(total - sum(r["ms"] for r in rows), 3), "ops": rows}


# ─── the headline: FLUX.1 step at 1024^2, Ulysses over the N ranks ──────────────────────

def flux_config(world: int) -> dict:
    return {"workload": "flux1_schnell_arch_dit_1024px", "tokens": FLUX_TXT + (FLUX_SIDE // 16) ** 2,
            "image_tokens": (FLUX_SIDE // 16) ** 2, "text_tokens": FLUX_TXT, "batch": 1, "hidden": 3072, "heads": 24,
            "head_dim": 128, "blocks": "19 double + 38 single", "linears": "W8A8, ConvRot 256",
            "attention": "INT8, reference quant mode", "sampler": "euler, 4-step schedule repeated, shift 1",
            "parallelism": (f"ulysses x{world}: tokens split over the ranks, NCCL all-to-all of q/k/v and "
                            "attention output" if world > 1 else "one GPU"),
            "l2": "~12 GB of weights streamed per step (> 126 MB L2)", "graph": "one CUDA graph per forward"}


# GPU kernel launches of this library per runner op (attention in the reference's quant mode:
# k_stats, k_sum, K codes, Q codes, main kernel; one more with the key-range split's combine)
_LAUNCHES_PER_OP = {"gemm": 1, "quant": 1, "ln_mod_quant": 1, "quant_seg": 1, "qk_norm_rope": 1, "attention": 5}


class _EulerSteps:
    """Euler flow-matching steps (src/diffucore/pipelines/_flux.py:226-236) on a captured forward:
    step i uses sigma index i % n of the n-step schedule and the latent restarts at x0 whenever
    i % n == 0, so any number of steps repeats the same sample. Allocation-free per step."""

    def __init__(self, fn, x0, sigmas):
        import torch
        self.fn, self.x0 = fn, x0
        self.x, self.tmp = x0.clone(), torch.empty_like(x0)
        self.n = len(sigmas) - 1
        self.ts = [torch.full((1,), float(sigmas[i]), device=x0.device, dtype=x0.dtype) for i in range(self.n)]
        self.dts = [(sigmas[i + 1] - sigmas[i]).to(x0.dtype).to(x0.device) for i in range(self.n)]

    def step(self, i: int) -> None:
        import torch
        k = i % self.n
        if k == 0:
            self.x.copy_(self.x0)
        v = self.fn(self.x, self.ts[k])
        torch.mul(v, self.dts[k], out=self.tmp)          # x + (sigma_next - sigma) v, rounded as euler_sample
        self.x.add_(self.tmp)


def _gather_rows(x, world: int):
    """This rank's rows of x [n, C] gathered on every rank in rank order (ranks may own different
    row counts)."""
    import torch
    import torch.distributed as dist
    n = torch.tensor([x.shape[0]], device=x.device, dtype=torch.int64)
    counts = [torch.zeros_like(n) for _ in range(world)]
    dist.all_gather(counts, n)
    mx = max(int(c) for c in counts)
    buf = torch.zeros(mx, x.shape[1], device=x.device, dtype=x.dtype)
    buf[: x.shape[0]] = x
    bufs = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(bufs, buf)
    return torch.cat([b[: int(c)] for b, c in zip(bufs, counts)])


def bench_flux_headline(args, world, rank, dev, peaks, sampler) -> dict:
    """The headline step (see the module docstring). Returns the line's headline keys plus
    `details` (everything measured)."""
    import torch
    import torch.distributed as dist
    from diffucore_b200 import _attention, _lib, flux
    t0 = time.perf_counter()
    model = flux.build_flux(flux.FluxConfig(), seed=0, device=dev, group=256)
    _attention.set_attention_backend(model, "int8_turing")
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    pg = dist.group.WORLD if world > 1 else None
    lat = FLUX_SIDE // 8
    n_img = (lat // 2) ** 2
    L = FLUX_TXT + n_img
    runner = flux.FluxRunner(model, FLUX_TXT, n_img, process_group=pg, device=dev, attn_mode=_lib.MODE_REF)
    runner.set_positions(flux.img_ids(lat, lat, 2, device=dev), flux.txt_ids(FLUX_TXT, device=dev))
    g = torch.Generator(device=dev).manual_seed(1)
    x_all = flux.patchify(torch.randn(1, 16, lat, lat, generator=g, device=dev)).to(torch.bfloat16)[0]
    txt_all = torch.randn(FLUX_TXT, 4096, generator=g, device=dev).to(torch.bfloat16)
    y = torch.randn(1, 768, generator=g, device=dev).to(torch.bfloat16)
    i0, i1 = runner.img_rows
    r0 = runner.rows[0]
    x0, txt = x_all[i0:i1].contiguous(), txt_all[r0: r0 + runner.t_loc].contiguous()
    sigmas = flux.flow_schedule(FLUX_STEPS, 1.0)
    graph = flux.FluxGraph(runner, x0, txt, y)
    eul = _EulerSteps(graph, x0, sigmas)
    for i in range(args.warmup):
        eul.step(i)
    torch.cuda.synchronize()
    # clock soak: the same steps right before the timed region, sampled with it (a fixed count, so
    # every rank runs the same collectives)
    sampler.start()
    for i in range(16):
        eul.step(i)
    torch.cuda.synchronize()
    start, end = _events(2)
    _barrier(world)
    torch.cuda.synchronize()
    start.record()
    for i in range(args.steps):
        eul.step(i)
    end.record()
    torch.cuda.synchronize()
    _barrier(world)
    clocks = sampler.stop()
    s_step = _max_over_ranks(start.elapsed_time(end) * 1e-3 / args.steps, world)
    finite = bool(torch.isfinite(eul.x).all())

    # end to end through the public API: every step copies its latent and text rows in from pinned
    # host memory and its updated latent back (same stream: each copy-in follows the last copy-out)
    hx0, hx = x0.cpu().pin_memory(), x0.cpu().pin_memory()
    htxt = txt.cpu().pin_memory()
    dx, dtxt = torch.empty_like(x0), torch.empty_like(txt)
    tmp = torch.empty_like(x0)

    def e2e_step(i):
        k = i % eul.n
        dx.copy_(hx0 if k == 0 else hx, non_blocking=True)
        dtxt.copy_(htxt, non_blocking=True)
        v = graph(dx, eul.ts[k], dtxt)
        torch.mul(v, eul.dts[k], out=tmp)
        dx.add_(tmp)
        hx.copy_(dx, non_blocking=True)

    for i in range(max(3, args.warmup)):
        e2e_step(i)
    torch.cuda.synchronize()
    es, ee = _events(2)
    _barrier(world)
    torch.cuda.synchronize()
    es.record()
    for i in range(args.steps):
        e2e_step(i)
    ee.record()
    torch.cuda.synchronize()
    _barrier(world)
    e2e_s = _max_over_ranks(es.elapsed_time(ee) * 1e-3 / args.steps, world)
    bi = (x0.numel() + txt.numel()) * 2
    bo = x0.numel() * 2
    if world > 1:
        tot = torch.tensor([bi, bo], device=dev, dtype=torch.float64)
        dist.all_reduce(tot)
        bi, bo = int(tot[0].item()), int(tot[1].item())
    e2e = {"value": e2e_s, "unit": "s/step", "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo,
           "steps": args.steps, "api": "FluxGraph + Euler update; pinned host latent/text in, latent out"}

    # per-op GPU time of one eager forward (events around every runner op): the dominant kernel's
    # achieved rate, the other hot kernels, and the launches per forward
    timed = flux.TimedOps()
    runner.ops = timed
    t_mid = torch.full((1,), 0.5, device=dev, dtype=torch.bfloat16)
    runner.forward(x0, txt, t_mid, y)
    rows = timed.summary()
    runner.ops = flux.CudaOps()
    gemm_ops = gemm_ms = attn_ms = 0.0
    attn_calls = 0
    launches = 0
    for r in rows:
        kind = r["op"].split(" ")[0]
        launches += _LAUNCHES_PER_OP.get(kind, 1) * r["calls"]
        if kind == "gemm":
            dims = dict(t.split("=") for t in r["op"].split(" ")[1:4])
            gemm_ops += 2.0 * int(dims["M"]) * int(dims["N"]) * int(dims["K"]) * r["calls"]
            gemm_ms += r["ms"]
        elif kind == "attention":
            attn_ms += r["ms"]
            attn_calls += r["calls"]
    hp = 24 // world
    attn_ops = attn_calls * 4.0 * L * L * 128 * hp
    peak = _int8_peak_tops(peaks)
    gemm_tops = gemm_ops / (gemm_ms * 1e-3) / 1e12 if gemm_ms else None
    attn_tops = attn_ops / (attn_ms * 1e-3) / 1e12 if attn_ms else None
    w = flux_work(L)
    compute_s = (w["linear_int8_ops"] + w["attn_int8_ops"]) / (peak * 1e12) + w["attn_bf16_ops"] / (peaks["bf16_tflops"] * 1e12)
    roof = compute_s / world
    a2a = 0.0
    if world > 1:
        Lr = L // world
        a2a = 57 * (Lr * 3 * 3072 + Lr * 3072) * 2 * (world - 1) / world / 770e9    # bytes sent per rank / peer copy
        roof = max(roof, a2a)

    # parity of the N-rank sample with one GPU's (rank 0 runs the same seeded 4-step sample alone).
    # The attention kernel is otherwise chosen by grid size (24 heads on one GPU, 24/N per rank)
    # and those kernels differ in summation order by ~1e-3 per call, which 57 blocks x 4 steps of
    # int8 requantization amplify; both sides run the same kernel here (eager, two-tile, no
    # key-range split) so that the check measures the distribution itself.
    parity = None
    if world > 1:
        with _env_set({"DC_ATTN_KERNEL": "two_tile", "DC_ATTN_SPLIT": "0"}):
            xs = flux.euler_sample(runner, x0, txt, y, sigmas)
            full = _gather_rows(xs, world)
            if rank == 0:
                one = flux.FluxRunner(model, FLUX_TXT, n_img, process_group=None, device=dev, attn_mode=_lib.MODE_REF)
                one.set_positions(flux.img_ids(lat, lat, 2, device=dev), flux.txt_ids(FLUX_TXT, device=dev))
                ref = flux.euler_sample(one, x_all, txt_all, y, sigmas).float()
                got = full.float()
                cos = torch.nn.functional.cosine_similarity(got.flatten().double(), ref.flatten().double(), dim=0).item()
                mad = (got - ref).abs().max().item()
                parity = {"max_abs": mad, "ref_max_abs": ref.abs().max().item(), "cos": cos,
                          "ok": bool(mad <= 2e-2 and cos >= 0.999),
                          "what": "final latent of the seeded 4-step sample, N ranks vs one GPU, same attention "
                                  "kernel on both (tolerance max-abs 2e-2, cos 0.999)"}
                del one, ref
        _barrier(world)
    del graph, runner
    torch.cuda.empty_cache()
    head = {
        "value": s_step, "ms_per_step": s_step * 1e3, "clocks": clocks, "e2e": e2e,
        "gpu_launches": launches * args.steps,
        "roofline": {"bound": "tensor", "achieved": gemm_tops, "peak": peak, "unit": "TOPS",
                     "frac": gemm_tops / peak if gemm_tops else None, "traffic": None,
                     "kernel": "gemm_w8a8_kernel, all block GEMMs of a forward, ops-weighted",
                     "peak_source": f"2 x bf16_tflops ({peaks['source']})",
                     "step": {"roofline_s": roof, "frac": roof / s_step}},
        "parity_vs_1gpu": parity, "finite": finite,
    }
    head["roofline"]["kernels"] = {"attention_flux": {
        "achieved": attn_tops, "frac": attn_tops / peak if attn_tops else None, "unit": "TOPS",
        "ms_per_call": attn_ms / max(attn_calls, 1), "heads_per_gpu": hp, "tokens": L}}
    head["details"] = {"build_s": build_s, "op_breakdown": rows, "roofline_s_per_step": roof,
                       "a2a_s_per_step_at_770GBps": a2a, "work_per_step_T": {k: v / 1e12 for k, v in w.items()}}
    return head


def bench_exchange(args, world: int, rank: int, dev) -> dict:
    """The Ulysses exchange alone: NCCL ``all_to_all_single`` of bf16 rows at the FLUX sizes per rank
    (q/k/v out: rows x 9216, attention output back: rows x 3072, rows = tokens / N at 1024^2 and
    2048^2), CUDA events over ``steps`` calls after ``warmup``, max over ranks."""
    import torch
    import torch.distributed as dist
    if world < 2:
        return {"skipped": "needs N > 1 ranks"}
    out = {}
    for side in (1024, 2048):
        rows = (FLUX_TXT + (side // 16) ** 2) // world
        for cols, what in ((9216, "qkv"), (3072, "attn_out")):
            x = torch.randn(rows * cols, device=dev).to(torch.bfloat16)
            y = torch.empty_like(x)
            for _ in range(args.warmup):
                dist.all_to_all_single(y, x)
            torch.cuda.synchronize()
            _barrier(world)
            s, e = _events(2)
            s.record()
            for _ in range(args.steps):
                dist.all_to_all_single(y, x)
            e.record()
            torch.cuda.synchronize()
            t = torch.tensor([s.elapsed_time(e) / args.steps], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            sent = rows * cols * 2 * (world - 1) / world
            out[f"{side}px_{what}_{rows}x{cols}"] = {"us": round(t.item() * 1e3, 1),
                                                      "gbs_sent_per_rank": round(sent / (t.item() * 1e-3) / 1e9, 1)}
            del x, y
    return {"what": "NCCL all_to_all_single, bf16, Ulysses exchange sizes per rank", "n_gpus": world, **out}


def bench_reference_gpu(args, dev) -> dict:
    """The reference's own GPU path for the two hot calls, timed on this GPU beside this library's:
    its W8A8 linear (Triton `_rot_quant_kernel` -> torch._int_mm (cuBLASLt) -> Triton
    `_rescale_kernel`, src/diffucore/models/_int8.py:158-168, :299-323) on config 1, and its INT8
    attention `fwd` (src/diffucore/kernels/int8_attn_sm80.cu:460-497, mma.sync, fp16 only) on
    config 2's shape in fp16, against this library's attention in the same (reference) quant mode.
    Both are the reference's unchanged code, staged / compiled into oracle/_ref/ by the checker
    recipe (oracle/build_ref.py); they are bars to compare with, never part of this library."""
    import torch
    from oracle import build_ref
    from diffucore_b200 import _int8, _lib, kernels
    out = {}
    warm, steps = max(3, args.warmup), max(10, min(args.steps, 50))

    def timeit(fn):
        for i in range(warm):
            fn(i)
        torch.cuda.synchronize()
        s, e = _events(2)
        _cpu_runahead()
        s.record()
        for i in range(steps):
            fn(i)
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / steps

    if build_ref.int8_available():
        ref = build_ref.load_int8()
        g = torch.Generator().manual_seed(0)
        lin = torch.nn.Linear(GEMM_K, GEMM_N, bias=True).to(torch.bfloat16)
        with torch.no_grad():
            lin.weight.copy_((torch.randn(GEMM_N, GEMM_K, generator=g) * 0.02).to(torch.bfloat16))
            lin.bias.copy_((torch.randn(GEMM_N, generator=g) * 0.01).to(torch.bfloat16))
        lin = lin.to(dev)
        ref_layer = ref.Int8Linear.from_linear(lin, group=0)
        our_layer = _int8.Int8Linear.from_linear(lin, group=0)
        xs = [torch.randn(GEMM_M, GEMM_K, generator=g).to(torch.bfloat16).to(dev) for _ in range(6)]
        with torch.no_grad():
            # bit-identity with the reference's GPU arithmetic (its Triton kernels divide with
            # div.full.f32); the timing below uses this library's default (correctly rounded) division
            prev = _int8.quant_division()
            _int8.set_quant_division("triton")
            try:
                same = bool(torch.equal(ref_layer(xs[0]), our_layer(xs[0])))
            finally:
                _int8.set_quant_division(prev)
            ref_ms = timeit(lambda i: ref_layer(xs[i % 6]))
            our_ms = timeit(lambda i: our_layer(xs[i % 6]))
            # the reference's three steps alone
            rq = [ref.quantize_activation(x, 0) for x in xs]
            accs = [ref.int_mm(q, ref_layer.weight) for q, _ in rq[:2]]
            parts = {"quantize_ms": timeit(lambda i: ref.quantize_activation(xs[i % 6], 0)),
                     "int_mm_ms": timeit(lambda i: ref.int_mm(rq[i % 6][0], ref_layer.weight)),
                     "rescale_ms": timeit(lambda i: ref.rescale(accs[i % 2], rq[i % 2][1], ref_layer.scale,
                                                                ref_layer.bias, torch.bfloat16))}
        out["w8a8_linear_config1"] = {"reference_ms": ref_ms, "ours_ms": our_ms, "speedup": ref_ms / our_ms,
                                      "bit_identical_triton_division": same, "reference_parts": parts,
                                      "reference_path": "Triton _rot_quant_kernel + torch._int_mm + Triton _rescale_kernel"}
        del rq, accs
        del xs
    else:
        out["w8a8_linear_config1"] = {"error": "reference _int8.py not staged in oracle/_ref"}
    if build_ref.available():
        mod = build_ref.load()
        g = torch.Generator(device=dev).manual_seed(2)
        sets = [tuple(torch.randn(B, S, H, D, generator=g, device=dev).half() for _ in range(3)) for _ in range(4)]
        plan = kernels.AttnPlan(B, H, S, S, D, torch.float16, _lib.MODE_REF, dev)
        o = torch.empty(B, S, H, D, device=dev, dtype=torch.float16)
        ref_ms = timeit(lambda i: mod.fwd(*sets[i % 4], D ** -0.5))
        our_ms = timeit(lambda i: plan(*sets[i % 4], o, D ** -0.5))
        a = mod.fwd(*sets[0], D ** -0.5).float().reshape(B, S, H, D)
        plan(*sets[0], o, D ** -0.5)
        cos = torch.nn.functional.cosine_similarity(a.flatten().double(), o.float().flatten().double(), dim=0).item()
        out["attention_config2_fp16_ref_mode"] = {
            "reference_ms": ref_ms, "ours_ms": our_ms, "speedup": ref_ms / our_ms,
            "reference_tops": ATTN_OPS / ref_ms / 1e9, "ours_tops": ATTN_OPS / our_ms / 1e9,
            "max_abs_vs_reference": (a - o.float()).abs().max().item(), "cos_vs_reference": cos,
            "reference_path": "int8_attn_sm80.cu fwd (mma.sync, compute_100 build)"}
        del sets
    else:
        out["attention_config2_fp16_ref_mode"] = {"error": "reference attention not built in oracle/_ref"}
    torch.cuda.empty_cache()
    return out


def bench_attention_config2(args, world, dev, peaks) -> dict:
    """BASELINE config 2 on its own: the INT8 attention (B=1, H=24, S=4608, D=128, bf16, block64),
    Q/K quantization + main kernel per step over rotating input sets; TOPS of the whole call and of
    the main kernel, its roofline against the INT8 peak and against its mixed ceiling (QK^T at the
    INT8 peak plus P.V at the bf16 peak), the reference quant mode's step, and the same call end to
    end with host buffers."""
    import torch
    from diffucore_b200 import _lib, kernels
    g = torch.Generator().manual_seed(0)
    sets = []
    for _ in range(4):
        q, k, v = (torch.randn(B, H, S, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
        sets.append((q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)))   # (B, L, H, D) views of bhld
    out = torch.empty(B, S, H, D, device=dev, dtype=torch.bfloat16)
    plan = kernels.AttnPlan(B, H, S, S, D, torch.bfloat16, _lib.MODE_BLOCK64, dev)
    t = bench_attention(args, world, _lib.MODE_BLOCK64, sets, plan, out)
    ref_plan = kernels.AttnPlan(B, H, S, S, D, torch.bfloat16, _lib.MODE_REF, dev)
    r = bench_attention(args, world, _lib.MODE_REF, sets, ref_plan, out)
    peak = _int8_peak_tops(peaks)
    main_tops = ATTN_OPS / (t["main_ms"] * 1e-3) / 1e12
    mixed_ms = (ATTN_OPS / 2 / (peak * 1e12) + ATTN_OPS / 2 / (peaks["bf16_tflops"] * 1e12)) * 1e3
    del sets, plan, ref_plan
    torch.cuda.empty_cache()
    return {"metric": ATTN_METRIC, "config": ATTN_CONFIG,
            "tops": ATTN_OPS / (t["total_ms"] / args.steps * 1e-3) / 1e12, "ms_per_call": t["total_ms"] / args.steps,
            "prep_ms": t["prep_ms"], "kernel_ms": t["main_ms"], "median_ms": t["median_ms"],
            "roofline": {"bound": "tensor", "achieved": main_tops, "peak": peak, "unit": "TOPS", "frac": main_tops / peak,
                         "traffic": TRAFFIC_ATTN, "kernel": "attn_int8_kernel<128, bf16>",
                         "mixed": {"target_ms": mixed_ms, "frac": mixed_ms / t["main_ms"]}},
            "ref_mode": {"ms_per_call": r["total_ms"] / args.steps, "prep_ms": r["prep_ms"], "kernel_ms": r["main_ms"],
                         "tops": ATTN_OPS / (r["total_ms"] / args.steps * 1e-3) / 1e12},
            "e2e": _guarded(bench_e2e, args, dev)}


def _compact(d, keys):
    """A few rounded numbers of a section dict (the long form goes to stderr)."""
    if not isinstance(d, dict):
        return d
    if "error" in d:
        return {"error": d["error"]}
    out = {}
    for k in keys:
        v = d
        for part in k.split("."):
            v = v.get(part) if isinstance(v, dict) else None
        if isinstance(v, float):
            v = round(v, 5 if abs(v) < 1 else 2)
        out[k.replace(".", "_")] = v
    return out


@contextlib.contextmanager
def _env_set(env: dict):
    """Environment variables set for the duration of the block (the library reads its kernel
    switches at each call); restored afterwards."""
    saved = {k: os.environ.get(k) for k in env}
    try:
        for k, v in env.items():
            os.environ[k] = v
        yield
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def _time_env(fn, env: dict, warmup: int, steps: int) -> float:
    """Mean device ms of fn(i) over `steps` calls with the environment variables in `env` set
    (the library reads its kernel switches at each call); restores the environment."""
    import torch
    saved = {k: os.environ.get(k) for k in env}
    try:
        for k, v in env.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
        for i in range(warmup):
            fn(i)
        torch.cuda.synchronize()
        st, en = _events(2)
        _cpu_runahead()
        st.record()
        for i in range(steps):
            fn(i)
        en.record()
        torch.cuda.synchronize()
        return st.elapsed_time(en) / steps
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


def bench_variants(args, dev, peaks) -> dict:
    """Kernel variants side by side on the same inputs (rotating sets larger than L2): the
    two-CTA GEMM (the default for wide GEMMs of 512+ rows without GELU) against the one-CTA kernel
    (DC_GEMM_PAIR=0) on config 1 and the FLUX block shapes, the two-tile attention against the
    single-tile one on config 2 in both quant modes, the key-range split attention (the default
    routing) against the unsplit dispatch (DC_ATTN_SPLIT=0) on one rank's share of FLUX's attention
    at 8 GPUs (3 heads, 4608 and 16896 tokens), and the packed-pair rotated row quantizers (the
    default) against the one-group kernels (DC_ROWQ_PAIR=0) on FLUX's rows. Times are device ms per
    call."""
    import torch
    from diffucore_b200 import _lib, kernels
    g = torch.Generator(device=dev).manual_seed(11)
    peak = _int8_peak_tops(peaks)
    warm, steps = max(3, args.warmup), max(10, min(args.steps, 100))
    out = {"unit": "ms per call", "peak_int8_tops": peak}
    gemms = {"config1 4096x3072x3072 bias": (4096, 3072, 3072, _lib.GELU_NONE, False),
             "flux qkv 4608x9216x3072": (4608, 9216, 3072, _lib.GELU_NONE, False),
             "flux mlp0 4608x12288x3072 gelu": (4608, 12288, 3072, _lib.GELU_TANH, False),
             "flux linear2 4608x3072x15360 gated": (4608, 3072, 15360, _lib.GELU_NONE, True)}
    for name, (M, N, K, gelu, gated) in gemms.items():
        nset = 3
        qs = [torch.randint(-127, 128, (M, K), generator=g, device=dev, dtype=torch.int8) for _ in range(nset)]
        w = torch.randint(-127, 128, (N, K), generator=g, device=dev, dtype=torch.int8)
        sx = torch.rand(M, generator=g, device=dev) * 1e-2 + 1e-4
        sw = torch.rand(N, generator=g, device=dev) * 1e-3 + 1e-5
        bias = (torch.randn(N, generator=g, device=dev) * 0.1).to(torch.bfloat16)
        gate = (torch.randn(N, generator=g, device=dev) * 0.5).to(torch.bfloat16) if gated else None
        ys = [torch.randn(M, N, generator=g, device=dev).to(torch.bfloat16) for _ in range(nset)]

        def fn(i, qs=qs, w=w, sx=sx, sw=sw, bias=bias, gate=gate, ys=ys, gelu=gelu):
            y = ys[i % len(ys)]
            kernels.gemm_w8a8_into(qs[i % len(qs)], w, sx, sw, bias, y, gelu=gelu, gate=gate,
                                   residual=y if gate is not None else None)

        ops = 2 * M * N * K
        row = {}
        for tag, env in (("one_cta", {"DC_GEMM_PAIR": "0"}), ("pair", {"DC_GEMM_PAIR": "1"})):
            ms = _time_env(fn, env, warm, steps)
            row[tag] = {"ms": round(ms, 4), "tops": round(ops / ms / 1e9, 1), "frac": round(ops / ms / 1e9 / peak, 3)}
        if not gated and gelu == _lib.GELU_NONE:
            # the same GEMM with the raw int32 accumulator as output (no rescale epilogue), and cuBLASLt's
            acc = torch.empty(M, N, device=dev, dtype=torch.int32)
            lib = _lib.load()

            def fn_i32(i, qs=qs, w=w, acc=acc):
                qq = qs[i % len(qs)]
                _lib.check(lib.dc_gemm_w8a8(kernels._ptr(qq), K, kernels._ptr(w), K, None, None, None,
                                            kernels._ptr(acc), N, _lib.DTYPE_I32, M, N, K, 0, kernels._stream(qq)))

            for tag, env in (("one_cta_int32_out", {"DC_GEMM_PAIR": "0"}), ("pair_int32_out", {"DC_GEMM_PAIR": "1"})):
                ms = _time_env(fn_i32, env, warm, steps)
                row[tag] = {"ms": round(ms, 4), "tops": round(ops / ms / 1e9, 1)}
            wt = w.t()
            ms = _time_env(lambda i, qs=qs, wt=wt: torch._int_mm(qs[i % len(qs)], wt), {}, warm, steps)
            row["cublaslt_int32_out"] = {"ms": round(ms, 4), "tops": round(ops / ms / 1e9, 1)}
            del acc
        out[name] = row
        del qs, w, ys
        torch.cuda.empty_cache()
    sets = []
    for _ in range(4):
        q, k, v = (torch.randn(B, H, S, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
        sets.append((q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)))
    o = torch.empty(B, S, H, D, device=dev, dtype=torch.bfloat16)
    for mode_name, mode in (("block64", _lib.MODE_BLOCK64), ("ref", _lib.MODE_REF)):
        plan = kernels.AttnPlan(B, H, S, S, D, torch.bfloat16, mode, dev)

        def fn(i, plan=plan):
            q, k, v = sets[i % len(sets)]
            plan(q, k, v, o, D ** -0.5)

        row = {}
        for tag, env in (("two_tile", {"DC_ATTN_KERNEL": "two_tile"}),
                         ("single_tile", {"DC_ATTN_KERNEL": "single_tile"})):
            ms = _time_env(fn, env, warm, steps)
            row[tag] = {"ms": round(ms, 4), "tops": round(ATTN_OPS / ms / 1e9, 1)}
        out[f"attention config2 {mode_name} (prep + main)"] = row
    # one rank's share of FLUX's attention on 8 GPUs (3 heads): default dispatch vs key-range split
    for L in (4608, 16896):
        hs = 3
        fsets = [tuple(torch.randn(1, L, hs, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
                 for _ in range(4)]
        fo = torch.empty(1, L, hs, D, device=dev, dtype=torch.bfloat16)
        nbytes = kernels.attn_workspace_layout(1, hs, L, L, D, _lib.MODE_REF)["total"]
        fws = torch.empty(nbytes, device=dev, dtype=torch.uint8)

        def fn(i, fsets=fsets, fo=fo, fws=fws):
            q, k, v = fsets[i % len(fsets)]
            kernels.attn_int8(q, k, v, D ** -0.5, _lib.MODE_REF, workspace=fws, out=fo)

        ops = 4 * hs * L * L * D
        row = {}
        for tag, env in (("unsplit", {"DC_ATTN_SPLIT": "0", "DC_ATTN_KERNEL": None}),
                         ("default", {"DC_ATTN_SPLIT": None, "DC_ATTN_KERNEL": None})):
            ms = _time_env(fn, env, warm, steps)
            row[tag] = {"ms": round(ms, 4), "tops": round(ops / ms / 1e9, 1)}
        out[f"attention 3 heads x {L} (FLUX rank share at 8 GPUs, mode ref)"] = row
        del fsets, fws
    out["row_quantizers"] = bench_rowq(args, dev, peaks)
    out["device_error"] = _lib.device_error()
    return out


def bench_rowq(args, dev, peaks) -> dict:
    """The row quantizers at FLUX row widths (bf16, group 256), same inputs rotating over sets
    larger than L2: the register-row kernel (the default), the packed-pair shared-memory kernels
    (DC_ROWQ_REG=0) and the one-group kernels (DC_ROWQ_REG=0 DC_ROWQ_PAIR=0); plain config-1 rows
    (no rotation) through the register-row kernel (DC_ROWQ_REG=2) against their default kernel.
    Device us per call and GB/s of 2 B read + 1 B written per element."""
    import torch
    from diffucore_b200 import _lib, kernels
    g = torch.Generator(device=dev).manual_seed(11)
    warm, steps = max(3, args.warmup), max(10, min(args.steps, 100))
    M, C, W = 4608, 3072, 15360
    xs = [torch.randn(M, C, generator=g, device=dev).to(torch.bfloat16) for _ in range(6)]
    shift = (0.1 * torch.randn(C, generator=g, device=dev)).to(torch.bfloat16)
    scale = (0.1 * torch.randn(C, generator=g, device=dev)).to(torch.bfloat16)
    wide = [torch.randn(M, W, generator=g, device=dev).to(torch.bfloat16) for _ in range(2)]
    mid = [torch.randn(4096, 12288, generator=g, device=dev).to(torch.bfloat16) for _ in range(3)]
    qbuf = torch.empty(M, W, device=dev, dtype=torch.int8)
    sbuf = torch.empty(M, device=dev, dtype=torch.float32)
    cases = (("ln_mod_quant 4608x3072 group 256",
              lambda i: kernels.ln_mod_quant(xs[i % 6], shift, scale, 256, qbuf[:, :C], sbuf), M * C),
             ("quant_rows 4608x3072 group 256",
              lambda i: kernels.quant_rows_into(xs[i % 6], 256, qbuf[:, :C], sbuf), M * C),
             ("quant_rows 4096x12288 group 256",
              lambda i: kernels.quant_rows_into(mid[i % 3], 256, qbuf[:4096, :12288], sbuf[:4096]), 4096 * 12288),
             ("quant_rows 4608x15360 group 256",
              lambda i: kernels.quant_rows_into(wide[i % 2], 256, qbuf, sbuf), M * W))
    out = {"unit": "us per call", "peak_hbm_gbs": peaks["hbm_gbs"]}
    variants = (("one_group", {"DC_ROWQ_REG": "0", "DC_ROWQ_PAIR": "0"}),
                ("pair", {"DC_ROWQ_REG": "0", "DC_ROWQ_PAIR": None}),
                ("register", {"DC_ROWQ_REG": None, "DC_ROWQ_PAIR": None}))
    for name, fn, elems in cases:
        row = {}
        for tag, env in variants:
            ms = _time_env(fn, env, warm, steps)
            row[tag] = {"us": round(ms * 1e3, 2), "gbs": round(elems * 3 / ms / 1e6, 1)}
        out[name] = row
    plain = [torch.randn(GEMM_M, GEMM_K, generator=g, device=dev).to(torch.bfloat16) for _ in range(6)]
    fn = lambda i: kernels.quant_rows_into(plain[i % 6], 0, qbuf[:GEMM_M, :GEMM_K], sbuf[:GEMM_M])  # noqa: E731
    row = {}
    for tag, env in (("default", {"DC_ROWQ_REG": None}), ("register", {"DC_ROWQ_REG": "2"})):
        ms = _time_env(fn, env, warm, steps)
        row[tag] = {"us": round(ms * 1e3, 2), "gbs": round(GEMM_M * GEMM_K * 3 / ms / 1e6, 1)}
    out[f"quant_rows {GEMM_M}x{GEMM_K} plain (config 1)"] = row
    out["device_error"] = _lib.device_error()
    return out


def bench_glue(args, dev, peaks) -> dict:
    """The FLUX block's HBM-bound glue kernels alone at 1024^2 shapes (4608 rows), GB/s of their
    algorithmic bytes against the measured HBM peak; inputs rotate over sets larger than L2."""
    import torch
    from diffucore_b200 import flux, kernels
    M, C, F = 4608, 3072, 12288
    g = torch.Generator(device=dev).manual_seed(3)
    nset = 3                   # 3 x 141 MB rows of the wide cases; 6 x 28 MB of the narrow ones (> 126 MB L2)
    xs = [torch.randn(M, C, generator=g, device=dev).to(torch.bfloat16) for _ in range(2 * nset)]
    big = [torch.randn(M, C + F, generator=g, device=dev).to(torch.bfloat16) for _ in range(nset)]
    qkv = [torch.randn(M, 3, 24, 128, generator=g, device=dev).to(torch.bfloat16) for _ in range(nset)]
    shift = (0.1 * torch.randn(C, generator=g, device=dev)).to(torch.bfloat16)
    scale = (0.1 * torch.randn(C, generator=g, device=dev)).to(torch.bfloat16)
    sc = (1 + 0.1 * torch.randn(128, generator=g, device=dev)).to(torch.bfloat16)
    pe = flux.rope_table(torch.cat([torch.zeros(512, 3), flux.img_ids(128, 128, 2)[0]]).to(dev), (16, 56, 56), 10_000)
    q = torch.empty(M, C + F, device=dev, dtype=torch.int8)
    s = torch.empty(M, device=dev, dtype=torch.float32)
    cases = {
        "ln_mod_quant K=3072 group 256": (lambda i: kernels.ln_mod_quant(xs[i % len(xs)], shift, scale, 256, q[:, :C], s),
                                          M * C * 3 + M * 4),
        "quant_rows K=15360 group 256": (lambda i: kernels.quant_rows_into(big[i % nset], 256, q, s), M * (C + F) * 3 + M * 4),
        "quant_rows K=15360 group 0": (lambda i: kernels.quant_rows_into(big[i % nset], 0, q, s), M * (C + F) * 3 + M * 4),
        "quant_rows K=3072 group 256": (lambda i: kernels.quant_rows_into(xs[i % len(xs)], 256, q[:, :C], s), M * C * 3 + M * 4),
        "qk_norm_rope 24 heads": (lambda i: kernels.qk_norm_rope(qkv[i % nset], sc, sc, pe), M * 2 * C * 2 * 2),
    }
    out = {"rows": M, "unit": "GB/s", "peak_hbm_gbs": peaks["hbm_gbs"]}
    for name, (fn, nbytes) in cases.items():
        for i in range(max(3, args.warmup)):
            fn(i)
        torch.cuda.synchronize()
        n = max(10, args.steps)
        st, en = _events(2)
        st.record()
        for i in range(n):
            fn(i)
        en.record()
        torch.cuda.synchronize()
        us = st.elapsed_time(en) * 1e3 / n
        out[name] = {"us": round(us, 2), "gbs": round(nbytes / us / 1e3, 1), "frac": round(nbytes / us / 1e3 / peaks["hbm_gbs"], 3)}
    return out


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--no-extras", action="store_true", help="the headline FLUX step only")
    ap.add_argument("--only", default="all",
                    choices=("all", "attention", "gemm", "flux", "glue", "sdxl", "variants", "rowq", "refgpu", "exchange"),
                    help="attention: BASELINE config 2 alone; gemm / flux: the config-1 W8A8 linear / the FLUX DiT "
                         "at 1024^2 and 2048^2; glue: the FLUX glue kernels; sdxl: the UNet; variants: kernel "
                         "variants against the defaults; rowq: the row quantizers; refgpu: the reference's own GPU "
                         "path against this library's; exchange: the Ulysses all-to-alls alone (N > 1)")
    ap.add_argument("--clocks-csv-dir", default=None,
                    help="also write the raw nvidia-smi clock samples of the timed region to this folder")
    ap.add_argument("--op-breakdown", action="store_true",
                    help="with --only flux: GPU time per runner op of one 1024^2 forward (CUDA events)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        return run_reference(args)

    import torch
    world, rank, local = _dist()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    peaks = _peaks()

    def finish(res) -> int:
        if rank == 0:
            print(json.dumps(res), flush=True)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return 0

    if args.only == "flux" and args.op_breakdown:
        return finish(flux_op_breakdown(dev))
    if args.only in ("glue", "sdxl", "variants", "rowq"):
        fn = {"glue": bench_glue, "sdxl": bench_sdxl, "variants": bench_variants, "rowq": bench_rowq}[args.only]
        return finish(fn(args, dev, peaks))
    if args.only == "exchange":
        return finish(bench_exchange(args, world, rank, dev))
    if args.only == "refgpu":
        return finish(bench_reference_gpu(args, dev))
    if args.only == "attention":
        return finish(bench_attention_config2(args, world, dev, peaks))
    if args.only in ("gemm", "flux"):
        return finish(bench_gemm(args, dev, peaks, cpu_baseline=rank == 0 and world == 1) if args.only == "gemm"
                      else bench_flux(args, world, rank, dev, peaks, cpu_baseline=rank == 0 and world == 1))

    sampler = ClockSampler(local, Path(args.clocks_csv_dir) / f"clocks_rank{rank}.csv" if args.clocks_csv_dir else None)
    head = bench_flux_headline(args, world, rank, dev, peaks, sampler)
    details = {"headline": head.pop("details")}
    line = {
        "metric": METRIC, "value": head["value"], "unit": "s/step", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": head["ms_per_step"], "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8 (GEMMs, QK^T) + bf16 (P.V, activations)",
        "data": "synthetic: seeded random bf16 weights, N(0,1) latent/text/pooled",
        "config": flux_config(world),
        "parity_vs_1gpu": head["parity_vs_1gpu"],
        "roofline": head["roofline"], "clocks": head["clocks"], "e2e": head["e2e"],
        "gpu_launches": head["gpu_launches"], "finite": head["finite"],
    }
    if rank == 0 and world == 1:
        if _host_gib_available() < HOST_GIB_FOR_CPU_BASELINES:
            line["cpu_baseline"] = {"error": f"skipped: under {HOST_GIB_FOR_CPU_BASELINES:.0f} GiB of host memory free"}
        else:
            line["cpu_baseline"] = _guarded(_cpu_flux_baseline)
    if not args.no_extras:
        kern = line["roofline"]["kernels"]
        extras = {}
        if world == 1:
            att = _guarded(bench_attention_config2, args, world, dev, peaks)
            details["attention_config2"] = att
            kern["attention_config2"] = _compact(att, ["tops", "kernel_ms", "prep_ms", "roofline.achieved",
                                                       "roofline.frac", "roofline.mixed.frac", "ref_mode.tops"])
            gem = _guarded(bench_gemm, args, dev, peaks, cpu_baseline=False)
            details["w8a8_linear_config1"] = gem
            kern["gemm_config1"] = _compact(gem, ["gemm.ms", "gemm.roofline.achieved", "gemm.roofline.frac",
                                                  "cublaslt_int_mm.ms", "cublaslt_int_mm.tops"])
            kern["quantizer_config1"] = _compact(gem, ["quantizer.ms", "quantizer.roofline.achieved",
                                                       "quantizer.roofline.frac"])
            ref_gpu = _guarded(bench_reference_gpu, args, dev)
            details["reference_gpu"] = ref_gpu
            extras["reference_gpu"] = {k: _compact(v, ["reference_ms", "ours_ms", "speedup",
                                                       "bit_identical_triton_division", "cos_vs_reference"])
                                       for k, v in ref_gpu.items()} if "error" not in ref_gpu else ref_gpu
        fl = _guarded(bench_flux, args, world, rank, dev, peaks, sides=(2048,))
        details["flux_2048"] = fl
        extras["flux_2048"] = _compact(fl, ["2048px.s_per_step", "2048px.frac_of_roofline", "2048px.finite"])
        if world == 1:
            torch.cuda.empty_cache()
            sd = _guarded(bench_sdxl, args, dev, peaks, cpu_baseline=rank == 0)
            details["sdxl_unet"] = sd
            extras["sdxl_unet"] = _compact(sd, ["s_per_step", "cpu_baseline.value", "finite"])
        line["extras"] = extras
    if rank == 0:
        print("bench details: " + json.dumps(details), file=sys.stderr, flush=True)
    return finish(line)


if __name__ == "__main__":
    sys.exit(main())
