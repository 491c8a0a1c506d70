"""Torch restatement of the steps FluxRunner launches, for testing the runner's host logic
(buffer layouts, the Ulysses row/head exchange, the per-rank text/image split) on CPU with gloo.

Each op computes what the reference model computes at that point with its own torch ops
(src/diffucore/models/flux_dit.py: LayerNorm + modulation :282, QKNorm/RMSNorm :129-151, apply_rope
:179-184, SDPA attention :187-190, gated residuals :302-305; src/diffucore/models/_int8.py:
quantize_activation via `_rotate` + `_quantize_rows`, int_mm, rescale) and writes it into the
same buffer layout the sm_100a kernel would (column-block send layout, strided outputs,
in-place residuals). Test infrastructure only.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from diffucore_b200._int8 import _quantize_rows, _rotate


def _quant(x: torch.Tensor, group: int, q: torch.Tensor, s: torch.Tensor) -> None:
    codes, scale = _quantize_rows(_rotate(x.float(), group))
    q.copy_(codes)
    s.copy_(scale)


class TorchOps:
    def ln_mod_quant(self, x, shift, scale, group, q, s):
        y = (1 + scale) * F.layer_norm(x, (x.shape[-1],), eps=1e-6) + shift
        _quant(y, group, q, s)

    def quant(self, x, group, q, s):
        _quant(x, group, q, s)

    def quant_seg(self, recv, x2, group, q, s):
        parts = list(recv.unbind(0))
        if x2 is not None:
            parts.append(x2)
        _quant(torch.cat(parts, dim=1), group, q, s)

    def gemm(self, q, sx, lin, out, *, ldo=None, gelu=0, gate=None, residual=None, col_block=0, block_stride=0):
        acc = (q.double() @ lin.weight.double().T).to(torch.int32)          # exact int32
        dtype = out.dtype
        y = (acc.float() * (sx.float()[:, None] * lin.scale.float()[None, :])).to(dtype)
        if lin.bias is not None:
            y = y + lin.bias.to(dtype)
        if gelu == 1:
            y = F.gelu(y)
        elif gelu == 2:
            y = F.gelu(y, approximate="tanh")
        if residual is not None:
            y = residual + gate * y
        M, N = y.shape
        if col_block:
            nb = N // col_block
            dst = out.as_strided((nb, M, col_block), (block_stride, ldo, 1))
            dst.copy_(y.view(M, nb, col_block).transpose(0, 1))
        elif ldo is not None and out.dim() == 1:
            out.as_strided((M, N), (ldo, 1)).copy_(y)
        else:
            out.copy_(y)

    def qk_norm_rope(self, qkv, q0, k0, q1, k1, split_row, pe):
        L = qkv.shape[0]

        def rms(x, scale):
            xf = x.float()
            rrms = torch.rsqrt(torch.mean(xf ** 2, dim=-1, keepdim=True) + 1e-6)
            return (xf * rrms).to(x.dtype) * scale

        def rope(x):
            xr = x.float().reshape(*x.shape[:-1], -1, 1, 2)
            f = pe[:, None]                                   # [L, 1, D/2, 2, 2]
            out = f[..., 0] * xr[..., 0] + f[..., 1] * xr[..., 1]
            return out.reshape(*x.shape).type_as(x)

        for which, (s0, s1) in ((0, (q0, q1)), (1, (k0, k1))):
            x = qkv[:, which]
            lo = rms(x[:split_row], s0) if split_row > 0 else x[:0]
            hi = rms(x[split_row:], s1) if split_row < L else x[:0]
            qkv[:, which] = rope(torch.cat([lo, hi], dim=0))

    def attention(self, q, k, v, out, sm_scale, backend, mode, workspace):
        o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2), scale=sm_scale)
        out.copy_(o.transpose(1, 2))
