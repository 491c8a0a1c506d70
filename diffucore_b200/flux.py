"""FLUX.1-architecture DiT on the B200 kernels of this package: the caller whose per-step time
the INT8 hot path sets (src/diffucore/models/flux_dit.py, sampled by
src/diffucore/pipelines/_flux.py:226-236).

Two parts:

* :class:`Flux` — the parameter container, with the reference's module and state-dict names
  (BFL's ``img_in``, ``double_blocks.N.img_attn.qkv``, ``single_blocks.N.linear1`` ...), so a
  FLUX.1 checkpoint or the reference's own ``Flux`` state dict loads as is, and the reference's
  ``quantize_linears`` turns its block linears into :class:`~diffucore_b200._int8.Int8Linear`.
* :class:`FluxRunner` — the forward pass as fused launches on persistent device buffers, one
  process per GPU. Every block linear is one tcgen05 W8A8 GEMM whose epilogue applies the rescale,
  bias, GELU-tanh or the gated residual ``x + gate * y`` in place; LayerNorm + AdaLN modulation
  are fused into the activation quantizer; QK-RMSNorm + RoPE run in place on the packed qkv rows;
  attention is the INT8 flash-attention kernel over strided views of those rows. With a process
  group of P ranks the sequence is split into P contiguous row ranges (Ulysses): linears run on
  the local rows, and an NCCL all-to-all before and after each attention trades rows for heads
  (24 / P heads per rank over the whole sequence). The qkv GEMM writes its output directly in the
  all-to-all's send layout and the projection's quantizer reads the receive layout in place.

The arithmetic of each fused step rounds where the reference's torch ops round (see the kernel
headers); the model-level result matches the reference ``Flux`` within the tolerance the tests
state. Weights are random-initialised (no checkpoint is needed for timing or parity).
"""

from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib, kernels
from ._int8 import GROUP, Int8Linear, adopt_int8_layers, int8_layers, quantize_linears


@dataclass
class FluxConfig:
    """FLUX.1 hyper-parameters (src/diffucore/models/flux_dit.py:28-50); defaults are FLUX.1
    [schnell] (no guidance embedder)."""
    in_channels: int = 64
    context_in_dim: int = 4096
    vec_in_dim: int | None = 768
    hidden_size: int = 3072
    mlp_ratio: float = 4.0
    num_heads: int = 24
    depth: int = 19
    depth_single_blocks: int = 38
    axes_dim: Sequence[int] = (16, 56, 56)
    theta: int = 10_000
    qkv_bias: bool = True
    guidance_embed: bool = False

    @property
    def head_dim(self) -> int:
        return self.hidden_size // self.num_heads

    @property
    def mlp_hidden(self) -> int:
        return int(self.hidden_size * self.mlp_ratio)


# ─── parameter containers (reference names; forward is FluxRunner's) ───────────────────

class MLPEmbedder(nn.Module):
    def __init__(self, in_dim: int, hidden: int):
        super().__init__()
        self.in_layer = nn.Linear(in_dim, hidden)
        self.out_layer = nn.Linear(hidden, hidden)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.out_layer(F.silu(self.in_layer(x)))


class RMSNorm(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.scale = nn.Parameter(torch.ones(dim))


class QKNorm(nn.Module):
    def __init__(self, dim: int):
        super().__init__()
        self.query_norm = RMSNorm(dim)
        self.key_norm = RMSNorm(dim)


class Modulation(nn.Module):
    def __init__(self, dim: int, double: bool):
        super().__init__()
        self.multiplier = 6 if double else 3
        self.lin = nn.Linear(dim, self.multiplier * dim)


class SelfAttention(nn.Module):
    def __init__(self, dim: int, num_heads: int, qkv_bias: bool):
        super().__init__()
        self.num_heads = num_heads
        self.qkv = nn.Linear(dim, 3 * dim, bias=qkv_bias)
        self.norm = QKNorm(dim // num_heads)
        self.proj = nn.Linear(dim, dim)


def _mlp(hidden: int, mlp_hidden: int) -> nn.Sequential:
    return nn.Sequential(nn.Linear(hidden, mlp_hidden), nn.GELU(approximate="tanh"), nn.Linear(mlp_hidden, hidden))


class DoubleStreamBlock(nn.Module):
    def __init__(self, cfg: FluxConfig):
        super().__init__()
        C = cfg.hidden_size
        self.attn_backend = "sdpa"       # stamped by _attention.set_attention_backend
        self.img_mod = Modulation(C, double=True)
        self.img_attn = SelfAttention(C, cfg.num_heads, cfg.qkv_bias)
        self.img_mlp = _mlp(C, cfg.mlp_hidden)
        self.txt_mod = Modulation(C, double=True)
        self.txt_attn = SelfAttention(C, cfg.num_heads, cfg.qkv_bias)
        self.txt_mlp = _mlp(C, cfg.mlp_hidden)


class SingleStreamBlock(nn.Module):
    def __init__(self, cfg: FluxConfig):
        super().__init__()
        C = cfg.hidden_size
        self.attn_backend = "sdpa"
        self.hidden_size = C
        self.mlp_hidden_dim = cfg.mlp_hidden
        self.linear1 = nn.Linear(C, 3 * C + cfg.mlp_hidden)
        self.linear2 = nn.Linear(C + cfg.mlp_hidden, C)
        self.norm = QKNorm(cfg.head_dim)
        self.modulation = Modulation(C, double=False)


class LastLayer(nn.Module):
    def __init__(self, hidden: int, out_channels: int):
        super().__init__()
        self.linear = nn.Linear(hidden, out_channels)
        self.adaLN_modulation = nn.Sequential(nn.SiLU(), nn.Linear(hidden, 2 * hidden))


class Flux(nn.Module):
    """FLUX.1 transformer parameters under the reference's names. ``forward`` runs one
    :class:`FluxRunner` on this process's GPU (built and cached per token count)."""

    def __init__(self, config: FluxConfig | None = None):
        super().__init__()
        cfg = config or FluxConfig()
        if sum(cfg.axes_dim) != cfg.head_dim:
            raise ValueError(f"axes_dim {tuple(cfg.axes_dim)} must sum to head_dim {cfg.head_dim}")
        self.config = cfg
        C = cfg.hidden_size
        self.img_in = nn.Linear(cfg.in_channels, C)
        self.time_in = MLPEmbedder(256, C)
        self.vector_in = MLPEmbedder(cfg.vec_in_dim, C) if cfg.vec_in_dim else None
        self.guidance_in = MLPEmbedder(256, C) if cfg.guidance_embed else None
        self.txt_in = nn.Linear(cfg.context_in_dim, C)
        self.double_blocks = nn.ModuleList(DoubleStreamBlock(cfg) for _ in range(cfg.depth))
        self.single_blocks = nn.ModuleList(SingleStreamBlock(cfg) for _ in range(cfg.depth_single_blocks))
        self.final_layer = LastLayer(C, cfg.in_channels)
        self._runners: dict = {}

    def block_linear_names(self) -> list[str]:
        """The token-wise linears that run W8A8 (qkv, proj, MLP of every block)."""
        names = []
        for i in range(len(self.double_blocks)):
            for s in ("img", "txt"):
                names += [f"double_blocks.{i}.{s}_attn.qkv", f"double_blocks.{i}.{s}_attn.proj",
                          f"double_blocks.{i}.{s}_mlp.0", f"double_blocks.{i}.{s}_mlp.2"]
        for i in range(len(self.single_blocks)):
            names += [f"single_blocks.{i}.linear1", f"single_blocks.{i}.linear2"]
        return names

    def forward(self, img: torch.Tensor, img_ids: torch.Tensor, txt: torch.Tensor, txt_ids: torch.Tensor,
                timesteps: torch.Tensor, y: torch.Tensor | None = None,
                guidance: torch.Tensor | None = None) -> torch.Tensor:
        """Velocity for image tokens ``img`` [B, Li, in_channels] (the reference signature,
        src/diffucore/models/flux_dit.py:410-447), single GPU. The runner takes one sample at a time;
        a batch runs its samples in turn (the reference's pipelines call it with B = 1)."""
        key = (txt.shape[1], img.shape[1])
        runner = self._runners.get(key)
        if runner is None:
            runner = FluxRunner(self, txt.shape[1], img.shape[1], device=img.device)
            self._runners[key] = runner

        def pick(t, b):                 # per-sample slice of a [B, ...] or broadcast [1, ...] tensor
            return None if t is None else (t[b:b + 1] if t.shape[0] > 1 else t)

        outs = []
        for b in range(img.shape[0]):
            runner.set_positions(pick(img_ids, b), pick(txt_ids, b))
            outs.append(runner.forward(img[b], txt[b if txt.shape[0] > 1 else 0], pick(timesteps, b), pick(y, b),
                                       pick(guidance, b)))
        return torch.stack(outs)


# ─── embeddings, positions, schedule (functions of the reference pipeline) ───────────────

def timestep_embedding(t: torch.Tensor, dim: int, max_period: int = 10_000, time_factor: float = 1000.0) -> torch.Tensor:
    """Sinusoidal embedding of ``time_factor * t`` (flux_dit.py:99-113): cos half then sin half,
    in t's dtype when t is floating point."""
    t = time_factor * t
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    args = t[:, None].float() * freqs[None]
    emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
    if dim % 2:
        emb = torch.cat([emb, torch.zeros_like(emb[:, :1])], dim=-1)
    return emb.to(t.dtype) if torch.is_floating_point(t) else emb


def rope_table(ids: torch.Tensor, axes_dim: Sequence[int], theta: int) -> torch.Tensor:
    """``[L, head_dim / 2, 2, 2]`` fp32 rotation of each rotary pair for positions ``ids``
    [L, n_axes] (flux_dit.py:154-175): per axis, angle = pos * theta^(-2i/dim) in float64, then
    [[cos, -sin], [sin, cos]]; the axes' pairs are concatenated in order."""
    parts = []
    for a, dim in enumerate(axes_dim):
        scale = torch.arange(0, dim, 2, dtype=torch.float64, device=ids.device) / dim
        omega = 1.0 / (theta ** scale)
        ang = ids[:, a].to(torch.float64)[:, None] * omega[None]
        c, s = torch.cos(ang), torch.sin(ang)
        parts.append(torch.stack([c, -s, s, c], dim=-1).view(ids.shape[0], dim // 2, 2, 2))
    return torch.cat(parts, dim=1).float().contiguous()


def img_ids(h: int, w: int, patch: int = 2, n_axes: int = 3, device=None) -> torch.Tensor:
    """Axial ids of the (h/p x w/p) patch grid: axis 1 = row, axis 2 = column
    (src/diffucore/pipelines/_flux.py:99-106)."""
    gh, gw = h // patch, w // patch
    ids = torch.zeros(gh, gw, n_axes, device=device)
    ids[..., 1] = torch.arange(gh, device=device)[:, None]
    ids[..., 2] = torch.arange(gw, device=device)[None, :]
    return ids.reshape(1, gh * gw, n_axes)


def txt_ids(length: int, n_axes: int = 3, device=None) -> torch.Tensor:
    """FLUX.1 text ids: all zero (src/diffucore/pipelines/_flux.py:109-113)."""
    return torch.zeros(1, length, n_axes, device=device)


def patchify(x: torch.Tensor, patch: int = 2) -> torch.Tensor:
    """[B, C, h, w] -> [B, (h/p)(w/p), C p p] (src/diffucore/pipelines/_flux.py:74-76)."""
    B, C, h, w = x.shape
    x = x.view(B, C, h // patch, patch, w // patch, patch).permute(0, 2, 4, 1, 3, 5)
    return x.reshape(B, (h // patch) * (w // patch), C * patch * patch)


def flow_schedule(steps: int, shift: float = 1.0, device=None) -> torch.Tensor:
    """sigma(t) = shift t / (1 + (shift - 1) t) at t = (N - i) / N, i = 0..N
    (src/diffucore/sampling/schedules.py:180-200)."""
    t = torch.linspace(1.0, 0.0, steps + 1, dtype=torch.float64)
    return (shift * t / (1 + (shift - 1) * t)).to(device=device, dtype=torch.float32)


@torch.no_grad()
def init_random_(model: nn.Module, seed: int = 0, device=None, std: float = 0.02, bias_std: float = 0.01,
                 dtype: torch.dtype = torch.bfloat16) -> nn.Module:
    """Seeded random weights, by parameter name in sorted order so any module with these names
    (this ``Flux`` or the reference's) gets the same values: weights N(0, std), biases
    N(0, bias_std), RMSNorm scales 1 + N(0, 0.1). ``device`` is where the generator runs
    (CPU draws are reproducible across machines; CUDA draws are fast for the full model)."""
    gen_dev = torch.device(device) if device is not None else torch.device("cpu")
    g = torch.Generator(device=gen_dev).manual_seed(seed)
    params = dict(model.named_parameters())
    for name in sorted(params):
        p = params[name]
        vals = torch.randn(p.shape, generator=g, device=gen_dev, dtype=torch.float32)
        if name.endswith(".scale"):
            vals = 1.0 + 0.1 * vals
        elif name.endswith("bias"):
            vals = bias_std * vals
        else:
            vals = std * vals
        p.data = vals.to(device=p.device if p.device.type != "meta" else gen_dev, dtype=dtype)
    return model


def from_state_dict(state_dict: dict, config: FluxConfig | None = None, device="cuda") -> Flux:
    """A ``Flux`` loaded from a FLUX.1 transformer state dict, plain or a ComfyUI ``int8_tensorwise``
    checkpoint: built on the meta device, every ``comfy_quant``-tagged linear adopted as an
    :class:`Int8Linear` (its ``weight_scale`` becomes ``scale_bits``), then a strict load, the
    reference loader's sequence (src/diffucore/bundle.py:301-305 for its DiTs)."""
    with torch.device("meta"):
        model = Flux(config)
    sd = dict(state_dict)
    layers = int8_layers(sd)
    if layers:
        sd = adopt_int8_layers(model, sd, layers)
    model.load_state_dict(sd, strict=True, assign=True)
    return model.to(device).eval()


def build_flux(cfg: FluxConfig | None = None, seed: int = 0, device="cuda", group: int = GROUP,
               init_device=None) -> Flux:
    """A random-initialised bf16 ``Flux`` on ``device`` with its block linears quantized to
    W8A8 by ``quantize_linears`` (ConvRot ``group``), as the reference's generic int8 path does
    (src/diffucore/models/_int8.py:496-503)."""
    with torch.device("meta"):
        model = Flux(cfg)
    model = model.to_empty(device=device)
    init_random_(model, seed, device=init_device if init_device is not None else device)
    quantize_linears(model, model.block_linear_names(), device, group=group)
    return model.eval()


# ─── kernels the runner launches (the test suite substitutes a torch restatement) ───────

class LinearW:
    """One W8A8 linear as the runner feeds it to the GEMM: int8 weight [N, K], fp32 scale [N],
    bias [N] in the model dtype (or None), ConvRot group."""

    def __init__(self, weight: torch.Tensor, scale: torch.Tensor, bias: torch.Tensor | None, group: int):
        self.weight, self.scale, self.bias, self.group = weight, scale, bias, group

    @classmethod
    def of(cls, lin: Int8Linear, dtype: torch.dtype, rows: slice | torch.Tensor | None = None) -> "LinearW":
        """``lin`` (optionally a subset or permutation of its output rows) as contiguous operands."""
        w, sc = lin.weight, lin.scale
        b = lin.bias.detach().to(dtype) if lin.bias is not None else None
        if rows is not None:
            w, sc = w[rows], sc[rows]
            b = b[rows] if b is not None else None
        return cls(w.contiguous(), sc.float().contiguous(), b.contiguous() if b is not None else None, lin.group)


class CudaOps:
    """The sm_100a kernels behind the runner's steps."""

    fuses_q8 = True      # qk_norm_rope can write the attention's Q codes (q8_workspace)

    def exchange(self, out, inp, pg):
        import torch.distributed as dist
        dist.all_to_all_single(out, inp, group=pg)

    def ln_mod_quant(self, x, shift, scale, group, q, s):
        kernels.ln_mod_quant(x, shift, scale, group, q, s)

    def quant(self, x, group, q, s):
        kernels.quant_rows_into(x, group, q, s)

    def quant_seg(self, recv, x2, group, q, s):
        kernels.quant_rows_seg(recv, x2, group, q, s)

    def gemm(self, q, sx, lin: LinearW, out, *, ldo=None, gelu=0, gate=None, residual=None, col_block=0,
             block_stride=0):
        kernels.gemm_w8a8_into(q, lin.weight, sx, lin.scale, lin.bias, out, ldo=ldo, gelu=gelu, gate=gate,
                               residual=residual, col_block=col_block, block_stride=block_stride)

    def qk_norm_rope(self, qkv, q0, k0, q1, k1, split_row, pe, q8_workspace=None):
        kernels.qk_norm_rope(qkv, q0, k0, pe, q1, k1, split_row, q8_workspace=q8_workspace,
                             write_q=q8_workspace is None)

    def attention(self, q, k, v, out, sm_scale, backend, mode, workspace, q_ready=False):
        if backend == "sdpa":
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               scale=sm_scale)
            out.copy_(o.transpose(1, 2))
        else:
            kernels.attn_int8(q, k, v, sm_scale, mode, workspace=workspace, out=out, q_ready=q_ready)


class TimedOps:
    """Wraps the runner's ops with CUDA events on the launching stream and sums GPU time per op
    kind and shape (a profiling aid: events between launches keep the launches in order but add
    a little time)."""

    def __init__(self, ops=None):
        self.ops = ops if ops is not None else CudaOps()
        self.events: list = []

    def _tag(self, name, args, kwargs):
        if name == "gemm":
            q, lin = args[0], args[2]
            extra = " gated" if kwargs.get("gate") is not None else (" gelu" if kwargs.get("gelu") else "")
            return f"gemm M={q.shape[0]} N={lin.weight.shape[0]} K={lin.weight.shape[1]}{extra}"
        if name in ("quant", "ln_mod_quant"):
            return f"{name} K={args[0].shape[1]}"
        if name == "quant_seg":
            return "quant_seg"
        return name

    def __getattr__(self, name):
        fn = getattr(self.ops, name)

        def timed(*args, **kwargs):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            out = fn(*args, **kwargs)
            e.record()
            self.events.append((self._tag(name, args, kwargs), s, e))
            return out
        return timed

    def summary(self) -> list[dict]:
        """[{op, calls, ms, us_per_call}] sorted by total time (synchronizes)."""
        torch.cuda.synchronize()
        agg: dict = {}
        for tag, s, e in self.events:
            n, ms = agg.get(tag, (0, 0.0))
            agg[tag] = (n + 1, ms + s.elapsed_time(e))
        rows = [{"op": k, "calls": n, "ms": round(ms, 3), "us_per_call": round(1e3 * ms / n, 1)}
                for k, (n, ms) in agg.items()]
        return sorted(rows, key=lambda r: -r["ms"])


def ulysses_qkv_order(hidden: int, heads: int, head_dim: int, P: int) -> torch.Tensor:
    """Output-row order of a fused qkv projection that groups the rows by destination rank:
    new row (p, s, j, d) = old row s * hidden + (p * heads/P + j) * head_dim + d, for q/k/v s,
    rank p and local head j. The GEMM then writes [P, rows, 3 * heads/P * head_dim] blocks, each
    one rank's share."""
    Hp = heads // P
    return torch.arange(3 * hidden).view(3, P, Hp, head_dim).permute(1, 0, 2, 3).reshape(-1)


class FluxRunner:
    """One FLUX forward on this rank's rows, as fused launches on buffers allocated once.

    ``process_group`` (size P) splits the L = n_txt + n_img tokens (text first) into P contiguous
    ranges of L / P rows; this rank owns ``rows`` = [r L/P, (r+1) L/P), of which the first
    ``n_txt_local`` are text tokens. Requires L % P == 0 and num_heads % P == 0.

    ``overlap_exchange`` (default: the environment variable ``DC_FLUX_OVERLAP=1``; off otherwise)
    starts a single-stream block's q/k/v all-to-all as soon as its qkv GEMM is done and runs the
    block's MLP GEMM while it is in flight (the collective runs on the communicator's own stream
    and the compute stream waits for it before QK-norm + RoPE), instead of exchanging after both
    GEMMs. Same results either way."""

    def __init__(self, model: Flux, n_txt: int, n_img: int, *, process_group=None, device=None,
                 attn_mode: int = _lib.MODE_REF, ops=None, overlap_exchange: bool | None = None):
        cfg = model.config
        self.model, self.cfg = model, cfg
        self.ops = ops if ops is not None else CudaOps()
        self.pg = process_group
        if process_group is not None:
            import torch.distributed as dist
            self.P, self.rank = dist.get_world_size(process_group), dist.get_rank(process_group)
        else:
            self.P, self.rank = 1, 0
        P = self.P
        self.device = torch.device(device) if device is not None else model.img_in.weight.device
        self.dtype = model.img_in.weight.dtype
        self.C, self.H, self.D, self.F = cfg.hidden_size, cfg.num_heads, cfg.head_dim, cfg.mlp_hidden
        self.Lt, self.Li = n_txt, n_img
        self.L = n_txt + n_img
        if self.L % P or self.H % P:
            raise ValueError(f"{self.L} tokens and {self.H} heads must both divide by {P} ranks")
        self.Lr, self.Hp = self.L // P, self.H // P
        r0 = self.rank * self.Lr
        self.rows = (r0, r0 + self.Lr)
        self.t_loc = max(0, min(self.Lt - r0, self.Lr))        # local text rows come first
        self.i_loc = self.Lr - self.t_loc
        self.img_rows = (max(r0 - self.Lt, 0), max(r0 - self.Lt, 0) + self.i_loc)   # image-token indices owned
        self.attn_mode = int(attn_mode)
        if overlap_exchange is None:
            overlap_exchange = os.environ.get("DC_FLUX_OVERLAP") == "1"
        self.overlap_exchange = bool(overlap_exchange) and P > 1
        self.sm_scale = self.D ** -0.5
        self._prepare_weights()
        self._allocate()
        self._pack_modulations()
        self.pe = None

    # -- setup ---------------------------------------------------------------------------
    def _prepare_weights(self):
        m, dt, P = self.model, self.dtype, self.P
        groups = set()
        order = ulysses_qkv_order(self.C, self.H, self.D, P).to(self.device) if P > 1 else None
        self.dw = []
        for blk in m.double_blocks:
            w = {}
            for s in ("img", "txt"):
                attn, mlp = getattr(blk, f"{s}_attn"), getattr(blk, f"{s}_mlp")
                for lin in (attn.qkv, attn.proj, mlp[0], mlp[2]):
                    if not isinstance(lin, Int8Linear):
                        raise TypeError("FluxRunner needs the block linears quantized (quantize_linears)")
                    groups.add(lin.group)
                w[f"{s}_qkv"] = LinearW.of(attn.qkv, dt, order)
                w[f"{s}_proj"] = LinearW.of(attn.proj, dt)
                w[f"{s}_mlp0"] = LinearW.of(mlp[0], dt)
                w[f"{s}_mlp2"] = LinearW.of(mlp[2], dt)
            self.dw.append(w)
        self.sw = []
        for blk in m.single_blocks:
            for lin in (blk.linear1, blk.linear2):
                if not isinstance(lin, Int8Linear):
                    raise TypeError("FluxRunner needs the block linears quantized (quantize_linears)")
                groups.add(lin.group)
            qkv_rows = order if order is not None else slice(0, 3 * self.C)
            self.sw.append({
                "qkv": LinearW.of(blk.linear1, dt, qkv_rows),
                "mlp": LinearW.of(blk.linear1, dt, slice(3 * self.C, 3 * self.C + self.F)),
                "out": LinearW.of(blk.linear2, dt),
            })
        if len(groups) > 1:
            raise ValueError(f"block linears mix ConvRot groups {sorted(groups)}")
        self.group = groups.pop() if groups else 0

    def _allocate(self):
        dev, dt = self.device, self.dtype
        Lr, L, C, F_, P = self.Lr, self.L, self.C, self.F, self.P
        self.Wd = 3 * self.Hp * self.D                        # one rank's qkv columns
        self.X = torch.zeros(Lr, C, device=dev, dtype=dt)     # residual stream, local rows
        self.codes = torch.empty(Lr * (C + F_), device=dev, dtype=torch.int8)
        self.scales = torch.empty(Lr, device=dev, dtype=torch.float32)
        self.send = torch.empty(P * Lr * self.Wd, device=dev, dtype=dt)            # [P, Lr, Wd]
        self.recv = torch.empty(L * self.Wd, device=dev, dtype=dt) if P > 1 else self.send   # [L, 3, Hp, D]
        self.O = torch.empty(L * self.Hp * self.D, device=dev, dtype=dt)           # [L, Hp, D]
        self.O_recv = torch.empty(Lr * C, device=dev, dtype=dt) if P > 1 else None  # [P, Lr, Hp D]
        self.Hbuf = torch.empty(Lr, F_, device=dev, dtype=dt)
        self.Cbuf = torch.empty(Lr, C + F_, device=dev, dtype=dt)
        backends = {b.attn_backend for b in list(self.model.double_blocks) + list(self.model.single_blocks)}
        self.workspace = None
        if any(b != "sdpa" for b in backends):
            lay = kernels.attn_workspace_layout(1, self.Hp, L, L, self.D, self.attn_mode) if self.device.type == "cuda" else None
            if lay is not None:
                self.workspace = torch.empty(lay["total"], device=dev, dtype=torch.uint8)

    def _mod_linears(self) -> list:
        m = self.model
        lins = []
        for blk in m.double_blocks:
            lins += [blk.img_mod.lin, blk.txt_mod.lin]
        lins += [blk.modulation.lin for blk in m.single_blocks]
        lins.append(m.final_layer.adaLN_modulation[1])
        return lins

    def _pack_modulations(self) -> None:
        """On CUDA: every block's AdaLN modulation linear (and the final layer's) stacked into one
        [sum N, hidden] weight, so a forward computes them all in one GEMV over silu(vec) instead of
        58 small ones (they depend on the timestep and pooled vector only). A copy (~6.5 GB for
        FLUX.1); the CPU path keeps the per-block linears."""
        self._mod_w = self._mod_b = None
        if self.device.type != "cuda":
            return
        lins = self._mod_linears()
        self._mod_w = torch.cat([l.weight.detach() for l in lins]).contiguous()
        self._mod_b = torch.cat([l.bias.detach() for l in lins]).contiguous()
        self._mod_sizes = [l.out_features for l in lins]

    def _modulations(self, sv: torch.Tensor) -> list:
        """Per block (double: img, txt; single; final) the modulation vector lin(silu(vec))."""
        if self._mod_w is not None:
            return list(torch.split(F.linear(sv, self._mod_w, self._mod_b)[0], self._mod_sizes))
        return [lin(sv)[0] for lin in self._mod_linears()]

    def set_positions(self, img_ids_: torch.Tensor, txt_ids_: torch.Tensor) -> None:
        """RoPE table for the whole sequence (text ids first), from [1, L*, n_axes] ids."""
        ids = torch.cat([txt_ids_[0], img_ids_[0]], dim=0).to(self.device)
        if ids.shape[0] != self.L:
            raise ValueError(f"ids cover {ids.shape[0]} tokens, runner expects {self.L}")
        self.pe = rope_table(ids, self.cfg.axes_dim, self.cfg.theta)

    # -- helpers -------------------------------------------------------------------------
    def _codes(self, rows: int, K: int, row0: int = 0) -> torch.Tensor:
        return self.codes[: self.Lr * K].view(self.Lr, K)[row0: row0 + rows]

    def _fuse_q8(self, blk) -> bool:
        """Whether the norm + RoPE pass emits the Q codes: INT8 attention in the reference quant
        mode on ops that support it (environment DC_FLUX_Q8=0 turns it off)."""
        return (getattr(self.ops, "fuses_q8", False) and blk.attn_backend == "int8_turing"
                and self.attn_mode == _lib.MODE_REF and self.workspace is not None
                and os.environ.get("DC_FLUX_Q8", "1") != "0")

    def _exchange(self, out: torch.Tensor, inp: torch.Tensor, async_op: bool = False):
        """All-to-all of ``inp`` into ``out``; with ``async_op`` the collective's handle (the caller
        waits on it before reading ``out`` or writing ``inp``). Blocking exchanges go through the
        ops object when it has an ``exchange`` (so a timing wrapper sees them)."""
        import torch.distributed as dist
        if not async_op and hasattr(self.ops, "exchange"):
            return self.ops.exchange(out, inp, self.pg)
        return dist.all_to_all_single(out, inp, group=self.pg, async_op=async_op)

    def _qkv_views(self):
        r4 = self.recv.view(self.L, 3, self.Hp, self.D)
        return r4, r4[:, 0].unsqueeze(0), r4[:, 1].unsqueeze(0), r4[:, 2].unsqueeze(0)

    def _qkv_gemm(self, codes, sx, lin: LinearW, row0: int):
        """qkv projection of local rows [row0, row0 + M) into the send layout."""
        Wd, Lr = self.Wd, self.Lr
        if self.P > 1:
            self.ops.gemm(codes, sx, lin, self.send[row0 * Wd:], ldo=Wd, col_block=Wd, block_stride=Lr * Wd)
        else:
            self.ops.gemm(codes, sx, lin, self.send[row0 * Wd:], ldo=Wd)

    def _attend(self, blk, q0, k0, q1, k1, split_row, out4, exchanged: bool = False):
        """Exchange q/k/v (unless the caller already did), norm + RoPE, attention into ``out4``
        (1, L, Hp, D), exchange back."""
        if self.P > 1 and not exchanged:
            self._exchange(self.recv, self.send)
        r4, q, k, v = self._qkv_views()
        if self._fuse_q8(blk):
            # the norm + RoPE pass writes the attention's Q codes; q itself is not written back
            self.ops.qk_norm_rope(r4, q0, k0, q1, k1, split_row, self.pe, q8_workspace=self.workspace)
            self.ops.attention(q, k, v, out4, self.sm_scale, blk.attn_backend, self.attn_mode, self.workspace,
                               q_ready=True)
        else:
            self.ops.qk_norm_rope(r4, q0, k0, q1, k1, split_row, self.pe)
            self.ops.attention(q, k, v, out4, self.sm_scale, blk.attn_backend, self.attn_mode, self.workspace)
        if self.P > 1:
            self._exchange(self.O_recv, self.O)

    # -- blocks --------------------------------------------------------------------------
    def _double(self, blk: DoubleStreamBlock, w: dict, img_mod: torch.Tensor, txt_mod: torch.Tensor) -> None:
        ops, X, C, F_, g = self.ops, self.X, self.C, self.F, self.group
        t, i, s = self.t_loc, self.i_loc, self.scales
        im = img_mod.view(6, C)     # shift1, scale1, gate1, shift2, scale2, gate2
        tm = txt_mod.view(6, C)
        parts = [(0, t, tm, "txt"), (t, i, im, "img")]
        for row0, n, mod, name in parts:
            if n:
                ops.ln_mod_quant(X[row0: row0 + n], mod[0], mod[1], g, self._codes(n, C, row0), s[row0: row0 + n])
                self._qkv_gemm(self._codes(n, C, row0), s[row0: row0 + n], w[f"{name}_qkv"], row0)
        ta, ia = blk.txt_attn.norm, blk.img_attn.norm
        if self.P > 1:
            out4 = self.O.view(1, self.L, self.Hp, self.D)
        else:
            out4 = self.O.view(1, self.L, self.H, self.D)
        self._attend(blk, ta.query_norm.scale, ta.key_norm.scale, ia.query_norm.scale, ia.key_norm.scale,
                     self.Lt, out4)
        if self.P > 1:
            ops.quant_seg(self.O_recv.view(self.P, self.Lr, self.Hp * self.D), None, g, self._codes(self.Lr, C), s)
        else:
            ops.quant(self.O.view(self.L, C), g, self._codes(self.Lr, C), s)
        for row0, n, mod, name in parts:
            if n:
                xs = X[row0: row0 + n]
                ops.gemm(self._codes(n, C, row0), s[row0: row0 + n], w[f"{name}_proj"], xs, gate=mod[2], residual=xs)
        for row0, n, mod, name in parts:
            if n:
                ops.ln_mod_quant(X[row0: row0 + n], mod[3], mod[4], g, self._codes(n, C, row0), s[row0: row0 + n])
                ops.gemm(self._codes(n, C, row0), s[row0: row0 + n], w[f"{name}_mlp0"], self.Hbuf[row0: row0 + n],
                         gelu=_lib.GELU_TANH)
        ops.quant(self.Hbuf, g, self._codes(self.Lr, F_), s)
        for row0, n, mod, name in parts:
            if n:
                xs = X[row0: row0 + n]
                ops.gemm(self._codes(n, F_, row0), s[row0: row0 + n], w[f"{name}_mlp2"], xs, gate=mod[5], residual=xs)

    def _single(self, blk: SingleStreamBlock, w: dict, modv: torch.Tensor) -> None:
        ops, X, C, F_, g, Lr, s = self.ops, self.X, self.C, self.F, self.group, self.Lr, self.scales
        mod = modv.view(3, C)  # shift, scale, gate
        ops.ln_mod_quant(X, mod[0], mod[1], g, self._codes(Lr, C), s)
        self._qkv_gemm(self._codes(Lr, C), s, w["qkv"], 0)
        # The MLP half reads the same codes and writes Cbuf, which the q/k/v exchange (send ->
        # recv) does not touch, so with overlap_exchange it runs while the exchange is in flight.
        work = self._exchange(self.recv, self.send, async_op=True) if self.overlap_exchange else None
        ops.gemm(self._codes(Lr, C), s, w["mlp"], self.Cbuf[:, C:], gelu=_lib.GELU_TANH)
        if work is not None:
            work.wait()
        if self.P > 1:
            out4 = self.O.view(1, self.L, self.Hp, self.D)
        else:
            out4 = self.Cbuf[:, :C].view(Lr, self.H, self.D).unsqueeze(0)
        nrm = blk.norm
        self._attend(blk, nrm.query_norm.scale, nrm.key_norm.scale, None, None, self.L, out4,
                     exchanged=work is not None)
        if self.P > 1:
            ops.quant_seg(self.O_recv.view(self.P, Lr, self.Hp * self.D), self.Cbuf[:, C:], g,
                          self._codes(Lr, C + F_), s)
        else:
            ops.quant(self.Cbuf, g, self._codes(Lr, C + F_), s)
        ops.gemm(self._codes(Lr, C + F_), s, w["out"], X, gate=mod[2], residual=X)

    # -- forward -------------------------------------------------------------------------
    @torch.no_grad()
    def forward(self, img: torch.Tensor, txt: torch.Tensor, timesteps: torch.Tensor, y: torch.Tensor | None = None,
                guidance: torch.Tensor | None = None) -> torch.Tensor:
        """Velocity [n_img_local, in_channels] for this rank's image tokens ``img``
        [n_img_local, in_channels] given its text tokens ``txt`` [n_txt_local, context_dim]
        (flux_dit.py:410-447; text rows precede image rows in the joint sequence)."""
        if self.pe is None:
            raise RuntimeError("call set_positions(img_ids, txt_ids) first")
        m, C, t = self.model, self.C, self.t_loc
        vec = m.time_in(timestep_embedding(timesteps, 256).to(self.dtype))
        if m.guidance_in is not None:
            if guidance is None:
                raise ValueError("guidance-distilled FLUX requires a `guidance` tensor")
            vec = vec + m.guidance_in(timestep_embedding(guidance, 256).to(self.dtype))
        if m.vector_in is not None:
            vec = vec + m.vector_in(y)
        sv = F.silu(vec)
        if t:
            self.X[:t] = m.txt_in(txt)
        if self.i_loc:
            self.X[t:] = m.img_in(img)
        mods = self._modulations(sv)
        nd = len(m.double_blocks)
        for bi, (blk, w) in enumerate(zip(m.double_blocks, self.dw)):
            self._double(blk, w, mods[2 * bi], mods[2 * bi + 1])
        for bi, (blk, w) in enumerate(zip(m.single_blocks, self.sw)):
            self._single(blk, w, mods[2 * nd + bi])
        fl = m.final_layer
        shift, scale = mods[-1].view(1, -1).chunk(2, dim=-1)
        xi = self.X[t:]
        h = (1 + scale) * F.layer_norm(xi, (C,), eps=1e-6) + shift
        return fl.linear(h)


class FluxGraph:
    """One captured CUDA graph of ``runner.forward``: the ~1000 launches of a FLUX forward (and,
    with Ulysses, its NCCL all-to-alls) replay as one graph launch, so the host no longer paces
    the GPU. Inputs are copied into static buffers before each replay; the returned velocity is a
    static buffer overwritten by the next replay. The runner's buffers are already persistent; the
    torch ops of the forward allocate from the graph's private pool."""

    def __init__(self, runner: FluxRunner, img: torch.Tensor, txt: torch.Tensor, y: torch.Tensor | None,
                 guidance: torch.Tensor | None = None):
        self.runner = runner
        self.img, self.txt = img.clone(), txt.clone()
        self.y = y.clone() if y is not None else None
        self.t = torch.zeros(1, device=img.device, dtype=img.dtype)
        self.guidance = guidance.clone() if guidance is not None else None
        side = torch.cuda.Stream(device=img.device)
        side.wait_stream(torch.cuda.current_stream(img.device))
        with torch.cuda.stream(side):
            for _ in range(2):                       # warm-up outside capture (torch requirement)
                runner.forward(self.img, self.txt, self.t, self.y, self.guidance)
        torch.cuda.current_stream(img.device).wait_stream(side)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.out = runner.forward(self.img, self.txt, self.t, self.y, self.guidance)

    def __call__(self, img: torch.Tensor, t: torch.Tensor, txt: torch.Tensor | None = None) -> torch.Tensor:
        if img.data_ptr() != self.img.data_ptr():
            self.img.copy_(img)
        if txt is not None and txt.data_ptr() != self.txt.data_ptr():
            self.txt.copy_(txt)
        self.t.copy_(t)
        self.graph.replay()
        return self.out


def euler_sample(runner, x: torch.Tensor, txt: torch.Tensor, y: torch.Tensor | None,
                 sigmas: torch.Tensor, guidance: torch.Tensor | None = None) -> torch.Tensor:
    """Euler flow-matching integration of this rank's image tokens ``x`` [n_img_local, C_in]:
    x += (sigma_next - sigma) v(x, sigma) per step (src/diffucore/pipelines/_flux.py:226-236).
    ``runner`` is a :class:`FluxRunner` or a :class:`FluxGraph` captured on it."""
    dt = x.dtype
    for i in range(len(sigmas) - 1):
        sigma, sigma_next = sigmas[i], sigmas[i + 1]
        t = torch.full((1,), float(sigma), device=x.device, dtype=dt)
        if isinstance(runner, FluxGraph):
            v = runner(x, t, txt)
        else:
            v = runner.forward(x, txt, t, y, guidance)
        x = x + (sigma_next - sigma).to(dt) * v
    return x
