"""SDXL-architecture UNet on this package's W8A8 linears and INT8 attention:
the caller src/diffucore/models/unet.py and its SD/SDXL pipeline's Euler sampler.

The module and state-dict names are the reference's (`input_blocks.N.1.transformer_blocks.M.attn1.to_q`
and so on), so the reference's UNet state dict loads as is. Inside every SpatialTransformer the
attention and feed-forward linears (`to_q`, `to_k`, `to_v`, `to_out.0`, `ff.net.0.proj`,
`ff.net.2`) run as :class:`~diffucore_b200._int8.Int8Linear` (W8A8 tcgen05 GEMM with the rescale
and bias in its epilogue); self-attention (`attn1`, head dim 64, 4096 / 1024 tokens at 1024^2)
runs the INT8 attention kernel, cross-attention to the 77 text tokens stays exact
(`attn2.is_selfattn = False`, so `set_attention_backend(model, "int8_turing")` stamps "sdpa" on
it). Convolutions, GroupNorm, LayerNorm and GEGLU's gate are torch ops in the model dtype (fp16).
When `to_q`, `to_k`, `to_v` are all W8A8 on the same input (self-attention), the normed
activation is quantized once and feeds the three GEMMs (the codes are the same ones each
projection would compute).

ConvRot rotation is off (group 0): SDXL's 640-wide level has in-features that are not multiples
of 256.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _attention
from ._int8 import Int8Linear, adopt_int8_layers, int8_layers, quantize_activation, quantize_linears


@dataclass
class UNetConfig:
    """SD / SDXL UNet hyper-parameters (src/diffucore/models/unet.py:20-47)."""
    in_channels: int = 4
    model_channels: int = 320
    out_channels: int = 4
    num_res_blocks: int = 2
    attention_resolutions: tuple = (4, 2, 1)
    channel_mult: tuple = (1, 2, 4, 4)
    num_heads: int = 8
    context_dim: int = 768
    transformer_depth: object = 1
    num_head_channels: int = -1
    adm_in_channels: int = 0
    use_linear_in_transformer: bool = False


def sdxl_unet_config() -> UNetConfig:
    """SDXL base: 3 levels (320/640/1280), transformer depth 0/2/10, head dim 64, 2048-d context,
    2816-d added conditioning, linear projections in the transformers."""
    return UNetConfig(channel_mult=(1, 2, 4), transformer_depth=(0, 2, 10), num_head_channels=64,
                      context_dim=2048, adm_in_channels=2816, use_linear_in_transformer=True)


def timestep_embedding(timesteps: torch.Tensor, dim: int, max_period: int = 10000) -> torch.Tensor:
    """LDM sinusoidal embedding, cos half then sin half (unet.py:54-61)."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(half, dtype=torch.float32, device=timesteps.device) / half)
    args = timesteps[:, None].float() * freqs[None]
    return torch.cat([torch.cos(args), torch.sin(args)], dim=-1)


class GroupNorm32(nn.GroupNorm):
    """GroupNorm computed in fp32, output in the input dtype."""

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return F.group_norm(x.float(), self.num_groups, self.weight.float(), self.bias.float(), self.eps).type(x.dtype)


class TimestepEmbedSequential(nn.Sequential):
    def forward(self, x, emb, context):
        for layer in self:
            if isinstance(layer, ResBlock):
                x = layer(x, emb)
            elif isinstance(layer, SpatialTransformer):
                x = layer(x, context)
            else:
                x = layer(x)
        return x


class ResBlock(nn.Module):
    def __init__(self, channels: int, emb_channels: int, out_channels: int):
        super().__init__()
        self.in_layers = nn.Sequential(GroupNorm32(32, channels), nn.SiLU(), nn.Conv2d(channels, out_channels, 3, padding=1))
        self.emb_layers = nn.Sequential(nn.SiLU(), nn.Linear(emb_channels, out_channels))
        self.out_layers = nn.Sequential(GroupNorm32(32, out_channels), nn.SiLU(), nn.Dropout(0.0),
                                        nn.Conv2d(out_channels, out_channels, 3, padding=1))
        self.skip_connection = nn.Conv2d(channels, out_channels, 1) if channels != out_channels else nn.Identity()

    def forward(self, x: torch.Tensor, emb: torch.Tensor) -> torch.Tensor:
        h = self.in_layers(x) + self.emb_layers(emb)[:, :, None, None]
        return self.skip_connection(x) + self.out_layers(h)


def _split_heads(t: torch.Tensor, b: int, heads: int, dim_head: int) -> torch.Tensor:
    return t.view(b, -1, heads, dim_head).transpose(1, 2)


class CrossAttention(nn.Module):
    def __init__(self, query_dim: int, context_dim: int, heads: int, dim_head: int, is_selfattn: bool):
        super().__init__()
        inner = heads * dim_head
        self.heads, self.dim_head = heads, dim_head
        self.is_selfattn = is_selfattn
        self.attn_backend = "sdpa"
        self.to_q = nn.Linear(query_dim, inner, bias=False)
        self.to_k = nn.Linear(context_dim, inner, bias=False)
        self.to_v = nn.Linear(context_dim, inner, bias=False)
        self.to_out = nn.Sequential(nn.Linear(inner, query_dim), nn.Dropout(0.0))

    def _qkv(self, x: torch.Tensor, context: torch.Tensor | None):
        lins = (self.to_q, self.to_k, self.to_v)
        if context is None and all(isinstance(m, Int8Linear) for m in lins) and len({m.group for m in lins}) == 1:
            # self-attention: one quantization of x feeds the three projections
            x2 = x.reshape(-1, x.shape[-1])
            q8, s8 = quantize_activation(x2, self.to_q.group)
            return tuple(m.matmul_quantized(q8, s8, x.dtype).view(*x.shape[:-1], -1) for m in lins)
        ctx = x if context is None else context
        return self.to_q(x), self.to_k(ctx), self.to_v(ctx)

    def forward(self, x: torch.Tensor, context: torch.Tensor | None = None) -> torch.Tensor:
        b = x.shape[0]
        q, k, v = self._qkv(x, context)
        q, k, v = (_split_heads(t, b, self.heads, self.dim_head) for t in (q, k, v))
        out = _attention.attention_bhld(q, k, v, self.attn_backend)
        return self.to_out(out)


class GEGLU(nn.Module):
    def __init__(self, dim_in: int, dim_out: int):
        super().__init__()
        self.proj = nn.Linear(dim_in, dim_out * 2)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        h, gate = self.proj(x).chunk(2, dim=-1)
        return h * F.gelu(gate)


class FeedForward(nn.Module):
    def __init__(self, dim: int, mult: int = 4):
        super().__init__()
        self.net = nn.Sequential(GEGLU(dim, dim * mult), nn.Dropout(0.0), nn.Linear(dim * mult, dim))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.net(x)


class BasicTransformerBlock(nn.Module):
    def __init__(self, dim: int, heads: int, context_dim: int):
        super().__init__()
        self.attn1 = CrossAttention(dim, dim, heads, dim // heads, is_selfattn=True)
        self.ff = FeedForward(dim)
        self.attn2 = CrossAttention(dim, context_dim, heads, dim // heads, is_selfattn=False)
        self.norm1, self.norm2, self.norm3 = nn.LayerNorm(dim), nn.LayerNorm(dim), nn.LayerNorm(dim)

    def forward(self, x: torch.Tensor, context: torch.Tensor) -> torch.Tensor:
        x = x + self.attn1(self.norm1(x))
        x = x + self.attn2(self.norm2(x), context)
        return x + self.ff(self.norm3(x))


class SpatialTransformer(nn.Module):
    def __init__(self, channels: int, heads: int, context_dim: int, depth: int, use_linear: bool):
        super().__init__()
        self.use_linear = use_linear
        self.norm = nn.GroupNorm(32, channels, eps=1e-6, affine=True)
        if use_linear:
            self.proj_in, self.proj_out = nn.Linear(channels, channels), nn.Linear(channels, channels)
        else:
            self.proj_in, self.proj_out = nn.Conv2d(channels, channels, 1), nn.Conv2d(channels, channels, 1)
        self.transformer_blocks = nn.ModuleList(BasicTransformerBlock(channels, heads, context_dim) for _ in range(depth))

    def forward(self, x: torch.Tensor, context: torch.Tensor) -> torch.Tensor:
        b, c, h, w = x.shape
        y = self.norm(x)
        if self.use_linear:
            y = self.proj_in(y.reshape(b, c, h * w).transpose(1, 2))
            for blk in self.transformer_blocks:
                y = blk(y, context)
            y = self.proj_out(y).transpose(1, 2).reshape(b, c, h, w)
        else:
            y = self.proj_in(y).reshape(b, c, h * w).transpose(1, 2)
            for blk in self.transformer_blocks:
                y = blk(y, context)
            y = self.proj_out(y.transpose(1, 2).reshape(b, c, h, w))
        return y + x


class Downsample(nn.Module):
    def __init__(self, channels: int):
        super().__init__()
        self.op = nn.Conv2d(channels, channels, 3, stride=2, padding=1)

    def forward(self, x):
        return self.op(x)


class Upsample(nn.Module):
    def __init__(self, channels: int):
        super().__init__()
        self.conv = nn.Conv2d(channels, channels, 3, padding=1)

    def forward(self, x):
        return self.conv(F.interpolate(x, scale_factor=2.0, mode="nearest"))


class UNetModel(nn.Module):
    """SD1.5 / SDXL UNet (reference names; src/diffucore/models/unet.py:265-402, without DeepCache)."""

    def __init__(self, config: UNetConfig | None = None):
        super().__init__()
        cfg = config or UNetConfig()
        self.config = cfg
        mc = cfg.model_channels
        ted = mc * 4
        self.time_embed = nn.Sequential(nn.Linear(mc, ted), nn.SiLU(), nn.Linear(ted, ted))
        self.label_emb = None
        if cfg.adm_in_channels > 0:
            self.label_emb = nn.Sequential(nn.Sequential(nn.Linear(cfg.adm_in_channels, ted), nn.SiLU(), nn.Linear(ted, ted)))
        seq = isinstance(cfg.transformer_depth, (list, tuple))
        if seq:
            depths = list(cfg.transformer_depth)
        else:
            depths, ds = [], 1
            for _ in cfg.channel_mult:
                depths.append(cfg.transformer_depth if ds in cfg.attention_resolutions else 0)
                ds *= 2
        mid_depth = cfg.transformer_depth[-1] if seq else cfg.transformer_depth

        def heads(ch):
            return ch // cfg.num_head_channels if cfg.num_head_channels > 0 else cfg.num_heads

        def transformer(ch, depth):
            return SpatialTransformer(ch, heads(ch), cfg.context_dim, depth, cfg.use_linear_in_transformer)

        self.input_blocks = nn.ModuleList([TimestepEmbedSequential(nn.Conv2d(cfg.in_channels, mc, 3, padding=1))])
        chans, ch = [mc], mc
        for level, mult in enumerate(cfg.channel_mult):
            for _ in range(cfg.num_res_blocks):
                layers = [ResBlock(ch, ted, mult * mc)]
                ch = mult * mc
                if depths[level] > 0:
                    layers.append(transformer(ch, depths[level]))
                self.input_blocks.append(TimestepEmbedSequential(*layers))
                chans.append(ch)
            if level != len(cfg.channel_mult) - 1:
                self.input_blocks.append(TimestepEmbedSequential(Downsample(ch)))
                chans.append(ch)
        self.middle_block = TimestepEmbedSequential(ResBlock(ch, ted, ch), transformer(ch, mid_depth), ResBlock(ch, ted, ch))
        self.output_blocks = nn.ModuleList()
        for level, mult in list(enumerate(cfg.channel_mult))[::-1]:
            for i in range(cfg.num_res_blocks + 1):
                layers = [ResBlock(ch + chans.pop(), ted, mult * mc)]
                ch = mult * mc
                if depths[level] > 0:
                    layers.append(transformer(ch, depths[level]))
                if level != 0 and i == cfg.num_res_blocks:
                    layers.append(Upsample(ch))
                self.output_blocks.append(TimestepEmbedSequential(*layers))
        self.out = nn.Sequential(GroupNorm32(32, ch), nn.SiLU(), nn.Conv2d(mc, cfg.out_channels, 3, padding=1))

    def int8_linear_names(self) -> list[str]:
        """The attention and feed-forward linears of every transformer block."""
        leaves = (".attn1.to_q", ".attn1.to_k", ".attn1.to_v", ".attn1.to_out.0", ".attn2.to_q", ".attn2.to_k",
                  ".attn2.to_v", ".attn2.to_out.0", ".ff.net.0.proj", ".ff.net.2")
        return [n for n, m in self.named_modules() if isinstance(m, nn.Linear) and n.endswith(leaves)]

    def forward(self, x: torch.Tensor, timesteps: torch.Tensor, context: torch.Tensor,
                y: torch.Tensor | None = None) -> torch.Tensor:
        emb = self.time_embed(timestep_embedding(timesteps, self.config.model_channels).to(x.dtype))
        if self.label_emb is not None:
            emb = emb + self.label_emb(y.to(x.dtype))
        hs, h = [], x
        for blk in self.input_blocks:
            h = blk(h, emb, context)
            hs.append(h)
        h = self.middle_block(h, emb, context)
        for blk in self.output_blocks:
            h = blk(torch.cat([h, hs.pop()], dim=1), emb, context)
        return self.out(h)


# ─── construction, schedule, sampler ────────────────────────────────────────────────────

@torch.no_grad()
def init_random_(model: nn.Module, seed: int = 0, device=None, dtype: torch.dtype = torch.float16) -> nn.Module:
    """Seeded random weights by parameter name (sorted): conv / linear weights N(0, 1/fan_in) (unit
    gain, so activations keep their scale through the depth), biases N(0, 0.01), norm weights
    1 + N(0, 0.05), norm biases N(0, 0.01)."""
    gen_dev = torch.device(device) if device is not None else torch.device("cpu")
    g = torch.Generator(device=gen_dev).manual_seed(seed)
    params = dict(model.named_parameters())
    norms = {n for n, m in model.named_modules() if isinstance(m, (nn.GroupNorm, nn.LayerNorm))}
    for name in sorted(params):
        p = params[name]
        vals = torch.randn(p.shape, generator=g, device=gen_dev, dtype=torch.float32)
        owner = name.rsplit(".", 1)[0]
        if owner in norms:
            vals = (1.0 + 0.05 * vals) if name.endswith("weight") else 0.01 * vals
        elif name.endswith("bias"):
            vals = 0.01 * vals
        else:
            fan_in = p[0].numel() if p.dim() > 1 else p.numel()
            vals = vals / math.sqrt(fan_in)
        p.data = vals.to(device=p.device if p.device.type != "meta" else gen_dev, dtype=dtype)
    return model


def from_state_dict(state_dict: dict, config: UNetConfig | None = None, device="cuda") -> UNetModel:
    """A ``UNetModel`` loaded from a UNet state dict, plain or a ComfyUI ``int8_tensorwise``
    checkpoint (tagged linears adopted as :class:`Int8Linear`), then a strict load; see
    :func:`diffucore_b200.flux.from_state_dict`."""
    with torch.device("meta"):
        model = UNetModel(config or sdxl_unet_config())
    sd = dict(state_dict)
    layers = int8_layers(sd)
    if layers:
        sd = adopt_int8_layers(model, sd, layers)
    model.load_state_dict(sd, strict=True, assign=True)
    return model.to(device).eval()


def build_sdxl_unet(cfg: UNetConfig | None = None, seed: int = 0, device="cuda", init_device=None,
                    dtype: torch.dtype = torch.float16) -> UNetModel:
    """Random-initialised fp16 SDXL UNet with its attention / FF linears quantized to W8A8 (group 0)
    and INT8 self-attention."""
    with torch.device("meta"):
        model = UNetModel(cfg or sdxl_unet_config())
    model = model.to_empty(device=device)
    init_random_(model, seed, device=init_device if init_device is not None else device, dtype=dtype)
    quantize_linears(model, model.int8_linear_names(), device, group=0)
    _attention.set_attention_backend(model, "int8_turing")
    return model.eval()


def sd_sigmas(steps: int, device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """(sigmas[steps + 1], timesteps[steps]) of SD's scaled-linear discrete schedule (betas
    linspace(sqrt(0.00085), sqrt(0.012), 1000)^2), timesteps spaced evenly from 999 to 0, final
    sigma 0."""
    betas = torch.linspace(0.00085 ** 0.5, 0.012 ** 0.5, 1000, dtype=torch.float64) ** 2
    ac = torch.cumprod(1.0 - betas, dim=0)
    all_sigmas = ((1 - ac) / ac).sqrt()
    ts = torch.linspace(999, 0, steps, dtype=torch.float64)
    lo, hi, frac = ts.floor().long(), ts.ceil().long(), ts - ts.floor()
    log_s = (1 - frac) * all_sigmas[lo].log() + frac * all_sigmas[hi].log()
    sigmas = torch.cat([log_s.exp(), torch.zeros(1, dtype=torch.float64)])
    return sigmas.float().to(device), ts.float().to(device)


@torch.no_grad()
def euler_cfg_sample(model: UNetModel, x: torch.Tensor, context: torch.Tensor, y: torch.Tensor,
                     steps: int, cfg_scale: float = 5.0) -> torch.Tensor:
    """Euler sampling of an epsilon-prediction UNet with classifier-free guidance as one batch of 2
    (context and y stacked [uncond, cond]): x_in = x / sqrt(sigma^2 + 1),
    eps = eps_u + cfg (eps_c - eps_u), x += (sigma_next - sigma) eps."""
    sigmas, ts = sd_sigmas(steps, x.device)
    x = x * sigmas[0]
    for i in range(steps):
        s, s_next = sigmas[i], sigmas[i + 1]
        x_in = (x / torch.sqrt(s * s + 1)).to(x.dtype).expand(2, *x.shape[1:])
        t = ts[i].expand(2)
        eps = model(x_in, t, context, y).float()
        e = eps[0:1] + cfg_scale * (eps[1:2] - eps[0:1])
        x = (x.float() + (s_next - s) * e).to(x.dtype)
    return x
