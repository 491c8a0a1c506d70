"""The reference's CPU (torch-op) path of the W8A8 linear, restated with torch ops — TEST
INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): the timed CPU baseline of BASELINE config 1 in
``bench.py`` and a second checker in ``tests/``.

Without a GPU the reference's ``Int8Linear.forward`` runs its torch-op branch
(src/diffucore/models/_int8.py:158-170 with ``_fast()`` False): ConvRot by an fp32 matmul with the
normalised Kronecker power of the 4x4 Hadamard (:64-84), per-row symmetric int8 (:87-97),
``torch._int_mm`` with M <= 16 padded to 32 rows (:200-207), then the rescale rounded to the model
dtype before the bias is added in that dtype (:313-323). Pinned by the config-1 SHA-256 of the
reference's own output (``tests/golden/config1_sha256.json``).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

_H4 = ((1, 1, 1, -1), (1, 1, -1, 1), (1, -1, 1, 1), (-1, 1, 1, 1))


def hadamard(n: int) -> torch.Tensor:
    """fp32 [n, n]: the Kronecker power of the 4x4 Hadamard above, divided by sqrt(n)."""
    h4 = torch.tensor(_H4, dtype=torch.float32)
    h = h4
    while h.shape[0] < n:
        h = torch.kron(h, h4)
    if h.shape[0] != n:
        raise ValueError(f"group {n} is not a power of 4")
    return h / n ** 0.5


def rotate(t: torch.Tensor, group: int) -> torch.Tensor:
    """fp32 ``t @ H`` over each ``group``-wide slice of the last dimension (identity for 0)."""
    if not group:
        return t
    rows = t.reshape(-1, t.shape[-1] // group, group)
    return (rows @ hadamard(group).to(t.device)).reshape(t.shape)


def quantize_rows(t: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(int8 codes, fp32 scale per row): scale = max(amax / 127, 1e-30), code = round(x / scale)
    (half to even) clamped to [-128, 127]."""
    t = t.float()
    scale = torch.clamp(t.abs().amax(dim=-1) / 127.0, min=1e-30)
    codes = torch.clamp(torch.round(t / scale[..., None]), -128, 127).to(torch.int8)
    return codes, scale


def int_mm(q: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """int32 q [M, K] . w [N, K]^T via torch._int_mm (rows padded to 32 when M <= 16)."""
    m = q.shape[0]
    if m <= 16:
        return torch._int_mm(F.pad(q, (0, 0, 0, 32 - m)), w.t())[:m]
    return torch._int_mm(q, w.t())


def rescale(acc: torch.Tensor, sx: torch.Tensor, sw: torch.Tensor, bias: torch.Tensor | None,
            dtype: torch.dtype) -> torch.Tensor:
    """dtype(acc * (sx[m] * sw[n])), then + dtype(bias) in dtype."""
    y = (acc.float() * (sx[:, None] * sw)).to(dtype)
    return y if bias is None else y + bias.to(dtype)


def int8_linear(x: torch.Tensor, wq: torch.Tensor, ws: torch.Tensor, bias: torch.Tensor | None,
                group: int = 0) -> torch.Tensor:
    """The torch-op forward of a W8A8 linear with int8 weight ``wq`` [N, K] and fp32 scales ``ws``."""
    x2 = x.reshape(-1, x.shape[-1])
    q, sx = quantize_rows(rotate(x2.float(), group))
    y = rescale(int_mm(q, wq), sx, ws, bias, x.dtype)
    return y.reshape(*x.shape[:-1], wq.shape[0])


def quantize_weight(w: torch.Tensor, group: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel int8 of a [N, K] weight after the rotation."""
    return quantize_rows(rotate(w.float(), group))


class FluxOps:
    """The reference's CPU path for each step the FLUX runner (``diffucore_b200.flux.FluxRunner``)
    launches, so the runner can time the reference's arithmetic on the host cores: the FLUX block
    math of src/diffucore/models/flux_dit.py (LayerNorm + modulation :282, QKNorm :129-151,
    apply_rope :179-184, SDPA attention :187-190 — the attention dispatch's CPU path, gated
    residuals :302-305, tanh-GELU MLP :236-239) with every block linear through the W8A8 torch-op
    path above (``rotate`` + ``quantize_rows``, ``int_mm`` = torch._int_mm, ``rescale``). Each
    op writes into the buffer layout the runner gives it (strided rows, column blocks, in-place
    residuals). Used as the timed CPU baseline of the FLUX line in ``bench.py``; ``tests/`` pins
    it to the reference's own FLUX output."""

    @staticmethod
    def _quant(x, group, q, s):
        codes, scale = quantize_rows(rotate(x.float(), group))
        q.copy_(codes)
        s.copy_(scale)

    def ln_mod_quant(self, x, shift, scale, group, q, s):
        self._quant((1 + scale) * F.layer_norm(x, (x.shape[-1],), eps=1e-6) + shift, group, q, s)

    def quant(self, x, group, q, s):
        self._quant(x, group, q, s)

    def quant_seg(self, recv, x2, group, q, s):
        parts = list(recv.unbind(0)) + ([x2] if x2 is not None else [])
        self._quant(torch.cat(parts, dim=1), group, q, s)

    def gemm(self, q, sx, lin, out, *, ldo=None, gelu=0, gate=None, residual=None, col_block=0, block_stride=0):
        y = rescale(int_mm(q, lin.weight), sx.float(), lin.scale.float(), lin.bias, out.dtype)
        if gelu == 1:
            y = F.gelu(y)
        elif gelu == 2:
            y = F.gelu(y, approximate="tanh")
        if residual is not None:
            y = residual + gate * y
        M, N = y.shape
        if col_block:
            nb = N // col_block
            out.as_strided((nb, M, col_block), (block_stride, ldo, 1)).copy_(y.view(M, nb, col_block).transpose(0, 1))
        elif ldo is not None and out.dim() == 1:
            out.as_strided((M, N), (ldo, 1)).copy_(y)
        else:
            out.copy_(y)

    def qk_norm_rope(self, qkv, q0, k0, q1, k1, split_row, pe):
        L = qkv.shape[0]

        def rms(x, scale):
            xf = x.float()
            return (xf * torch.rsqrt(torch.mean(xf ** 2, dim=-1, keepdim=True) + 1e-6)).to(x.dtype) * scale

        def rope(x):
            xr = x.float().reshape(*x.shape[:-1], -1, 1, 2)
            f = pe[:, None]
            return (f[..., 0] * xr[..., 0] + f[..., 1] * xr[..., 1]).reshape(*x.shape).type_as(x)

        for which, (s0, s1) in ((0, (q0, q1)), (1, (k0, k1))):
            x = qkv[:, which]
            lo = rms(x[:split_row], s0) if split_row > 0 else x[:0]
            hi = rms(x[split_row:], s1) if split_row < L else x[:0]
            qkv[:, which] = rope(torch.cat([lo, hi], dim=0))

    def attention(self, q, k, v, out, sm_scale, backend, mode, workspace):
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), scale=sm_scale)
        out.copy_(o.transpose(1, 2))


class CpuInt8Linear(torch.nn.Module):
    """An ``Int8Linear``'s forward off the GPU, as the reference runs it there (its torch-op
    branch, src/diffucore/models/_int8.py:158-170 with ``_fast()`` False): ``int8_linear`` above
    on the layer's int8 weight, fp32 scales, bias and ConvRot group."""

    def __init__(self, layer: torch.nn.Module):
        super().__init__()
        self.in_features, self.out_features, self.group = layer.in_features, layer.out_features, layer.group
        self.register_buffer("wq", layer.weight.detach())
        self.register_buffer("ws", layer.scale.detach().float())
        self.bias = layer.bias

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return int8_linear(x, self.wq, self.ws, self.bias, self.group)


def cpu_int8_linears_(model: torch.nn.Module) -> int:
    """Replace every ``Int8Linear`` of ``model`` with :class:`CpuInt8Linear`; returns the count."""
    names = [n for n, m in model.named_modules() if type(m).__name__ == "Int8Linear"]
    for name in names:
        head, _, leaf = name.rpartition(".")
        parent = model.get_submodule(head) if head else model
        setattr(parent, leaf, CpuInt8Linear(getattr(parent, leaf)))
    return len(names)
