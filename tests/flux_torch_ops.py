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

from oracle.torch_ref import FluxOps


class TorchOps(FluxOps):
    """The reference's torch ops for every runner step (oracle/torch_ref.py ``FluxOps``) with the
    int32 products formed in fp64 (exact at these sizes) instead of torch._int_mm, so the same
    restatement runs on CPU and GPU tensors alike."""

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
