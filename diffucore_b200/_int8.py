"""W8A8 linears on the B200: the module and free-function API of diffucore's
``diffucore.models._int8`` (src/diffucore/models/_int8.py), re-implemented over the sm_100a
kernels of this package.

Forward-path functions (``quantize_activation``, ``int_mm``, ``rescale``, ``int8_mlp``,
``Int8Linear.forward``) run on CUDA tensors through ``libdiffucore_b200.so`` and raise for
anything else: there is no CPU or Triton path. ``scaled_mm`` keeps the reference's contract and
returns None for a call its fused GEMM cannot take (so off the GPU the caller's int32 path raises). Load-time helpers (``quantize_weight``
on CPU, ``dequantize_weight``, LoRA's ``add_delta_``, the checkpoint plumbing) are tensor
bookkeeping done once per layer and use torch ops, as the reference does.

State-dict layout is the reference's: ``weight`` int8 [N, K], ``scale_bits`` int32 [N] (the fp32
per-row scale stored as raw bits so ``module.to(dtype)`` never rounds it), optional ``bias``,
and the ConvRot ``group`` (0 or 256). ComfyUI ``int8_tensorwise`` checkpoints adopt as-is.
"""

from __future__ import annotations

import json
import zlib

import torch
import torch.nn as nn

from . import _lib, kernels

GROUP = 256            # ConvRot group used when quantizing at load (_int8.py:44)
_FUSED_MIN_ROWS = 1    # the tcgen05 GEMM fuses the rescale at every M (reference: 32, _int8.py:49)
_H4 = ((1, 1, 1, -1), (1, 1, -1, 1), (1, -1, 1, 1), (-1, 1, 1, 1))
_hadamard_cache: dict = {}


def _library_error() -> str:
    try:
        _lib.load()
        return ""
    except _lib.NativeLibraryError as e:
        return str(e)


def int8_fast_available(device=None) -> bool:
    """Whether int8 layers run here: an sm_100 CUDA device and the native library
    (reference semantics: _int8.py:53-61)."""
    if not torch.cuda.is_available():
        return False
    device = torch.device(device) if device is not None else torch.device("cuda")
    if device.type != "cuda":
        return False
    return torch.cuda.get_device_capability(device) == (10, 0) and not _library_error()


# ─── ConvRot rotation and per-row quantization (load-time, torch ops) ───────────────────

def _hadamard(n: int, device, dtype=torch.float32) -> torch.Tensor:
    """Normalised ``n x n`` Hadamard: the Kronecker power of ``_H4`` divided by sqrt(n)
    (_int8.py:64-76). ``n`` must be a power of 4."""
    key = (n, str(device), dtype)
    cached = _hadamard_cache.get(key)
    if cached is not None:
        return cached
    base = torch.tensor(_H4, dtype=torch.float32)
    mat = base
    while mat.shape[0] < n:
        mat = torch.kron(mat, base)
    if mat.shape[0] != n:
        raise ValueError(f"ConvRot group must be a power of 4, got {n}")
    mat = (mat / n ** 0.5).to(device, dtype)
    _hadamard_cache[key] = mat
    return mat


def _rotate(t: torch.Tensor, group: int) -> torch.Tensor:
    """``t @ H`` on each ``group``-wide slice of the last dim; identity for group 0 (_int8.py:79-84)."""
    if not group:
        return t
    shape = t.shape
    grouped = t.reshape(-1, shape[-1] // group, group)
    return (grouped @ _hadamard(group, t.device, t.dtype)).reshape(shape)


def _quantize_rows(t: torch.Tensor, generator: torch.Generator | None = None):
    """Per-row symmetric int8 with torch ops: ``scale = max(amax / 127, 1e-30)``, codes
    ``rint(t / scale)`` or, with ``generator``, ``floor(t / scale + U[0, 1))`` (unbiased
    stochastic rounding for re-quantizing on-grid weights). _int8.py:87-97."""
    t = t.float()
    scale = torch.clamp(t.abs().amax(-1) / 127.0, min=1e-30)
    scaled = t / scale.unsqueeze(-1)
    if generator is None:
        scaled = torch.round(scaled)
    else:
        noise = torch.rand(scaled.shape, device=scaled.device, generator=generator)
        scaled = torch.floor(scaled + noise)
    return torch.clamp(scaled, -128, 127).to(torch.int8), scale


def quantize_weight(w: torch.Tensor, group: int = GROUP):
    """``(int8 [N, K], fp32 [N])`` for a weight ``[N, K]`` after ConvRot rotation
    (_int8.py:100-102). On CUDA this is the native per-row quantizer (the same arithmetic;
    with group 256 the rotation runs as this library's butterfly)."""
    if w.is_cuda:
        return kernels.quant_rows(w.detach(), group)
    return _quantize_rows(_rotate(w.float(), group))


def dequantize_weight(q: torch.Tensor, scale: torch.Tensor, group: int) -> torch.Tensor:
    """fp32 weight in the original basis (H is its own inverse), _int8.py:105-107."""
    return _rotate(q.float() * scale.unsqueeze(-1), group)


# ─── hot path ───────────────────────────────────────────────────────────────────────────

_QDIV = {"ieee": _lib.QDIV_IEEE, "triton": _lib.QDIV_FULL}


def set_quant_division(mode: str) -> None:
    """Which of the reference's quantizer arithmetics the activation codes reproduce, process-wide:
    ``"ieee"`` (default) rounds ``amax / 127`` and ``x / scale`` correctly, the reference's torch-op
    path as it runs on the CPU (_int8.py:87-97); ``"triton"`` divides as the reference's Triton
    kernels do on a GPU (``_store_quantized``, _int8.py:393-397). The two give the same codes except
    for one step at ~1.5e-4 of elements."""
    if mode not in _QDIV:
        raise ValueError(f"quant division must be one of {sorted(_QDIV)}, got {mode!r}")
    _lib.check(_lib.load().dc_set_quant_division(_QDIV[mode]))


def quant_division() -> str:
    code = _lib.load().dc_quant_division()
    return next(k for k, v in _QDIV.items() if v == code)


def quantize_activation(x2: torch.Tensor, group: int):
    """``(int8 [M, K], fp32 scale [M])``: rotate, then per-row int8 (_int8.py:299-310), as one
    HBM pass of the native quantizer."""
    return kernels.quant_rows(x2, group)


def int_mm(q: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """int32 ``q @ w.T`` on the tcgen05 tensor core (_int8.py:200-207); any M."""
    return kernels.gemm_w8a8(q, w, None, None, None, torch.int32)


def rescale(acc: torch.Tensor, sx: torch.Tensor, sw: torch.Tensor, bias, dtype) -> torch.Tensor:
    """``acc * sx[:, None] * sw[None, :] (+ bias)`` in ``dtype`` (_int8.py:313-323)."""
    return kernels.rescale(acc, sx, sw, bias, dtype)


def fused_gemm_applies(device) -> bool:
    """Whether the fused-rescale GEMM serves ``device``: every sm_100 device (_int8.py:250-255)."""
    device = torch.device(device)
    return device.type == "cuda" and int8_fast_available(device)


def fused_gemm_error(device) -> str:
    """"" when the fused GEMM is usable on ``device``, else why not (_int8.py:258-263)."""
    device = torch.device(device)
    if device.type != "cuda" or not torch.cuda.is_available():
        return "device is not CUDA"
    if torch.cuda.get_device_capability(device) != (10, 0):
        return "GPU is not sm_100 (B200/GB200)"
    return _library_error()


def scaled_mm(q: torch.Tensor, w: torch.Tensor, sx: torch.Tensor, sw: torch.Tensor, dtype: torch.dtype):
    """``dtype(q @ w.T * sx[:, None] * sw)`` in one kernel, rounded exactly like :func:`rescale`
    (_int8.py:266-276). Returns None, as the reference does, when the fused GEMM cannot take the
    call -- tensors off the GPU, or a dtype its epilogue does not write -- so the caller falls back
    to :func:`int_mm` + :func:`rescale` (which have no CPU path here and say so)."""
    if dtype not in (torch.float16, torch.bfloat16) or not q.is_cuda:
        return None
    return kernels.gemm_w8a8(q, w, sx, sw, None, dtype)


class Int8Linear(nn.Module):
    """``nn.Linear`` with int8 weights and per-token int8 activations (_int8.py:110-170)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = False, group: int = GROUP,
                 device=None):
        super().__init__()
        if group and in_features % group:
            raise ValueError(f"in_features {in_features} is not a multiple of the ConvRot group {group}")
        self.in_features, self.out_features, self.group = in_features, out_features, group
        self.register_buffer("weight", torch.empty(out_features, in_features, dtype=torch.int8, device=device))
        self.register_buffer("scale_bits", torch.empty(out_features, dtype=torch.int32, device=device))
        if bias:
            self.bias = nn.Parameter(torch.empty(out_features, device=device), requires_grad=False)
        else:
            self.bias = None

    @property
    def scale(self) -> torch.Tensor:
        return self.scale_bits.view(torch.float32)

    @classmethod
    def from_linear(cls, linear: nn.Linear, group: int = GROUP, device=None) -> "Int8Linear":
        device = device if device is not None else linear.weight.device
        q, s = quantize_weight(linear.weight.detach().to(device), group)
        layer = cls(linear.in_features, linear.out_features, linear.bias is not None, group, device=device)
        layer.weight.copy_(q)
        layer.scale_bits.copy_(s.view(torch.int32))
        if linear.bias is not None:
            layer.bias = nn.Parameter(linear.bias.detach().to(device), requires_grad=False)
        return layer

    def to_linear(self, dtype: torch.dtype) -> nn.Linear:
        lin = nn.Linear(self.in_features, self.out_features, bias=self.bias is not None, device="meta")
        lin.weight = nn.Parameter(dequantize_weight(self.weight, self.scale, self.group).to(dtype),
                                  requires_grad=False)
        if self.bias is not None:
            lin.bias = nn.Parameter(self.bias.detach().to(dtype), requires_grad=False)
        return lin

    @torch.no_grad()
    def add_delta_(self, delta: torch.Tensor, seed: int) -> None:
        """``W += delta`` re-quantized with seeded stochastic rounding (_int8.py:148-156): the
        weights sit on the int8 grid, so nearest rounding would erase sub-step deltas."""
        w = self.weight.float() * self.scale.unsqueeze(-1) + _rotate(delta.float(), self.group)
        q, s = _quantize_rows(w, torch.Generator(device=w.device).manual_seed(seed))
        self.weight.copy_(q)
        self.scale_bits.copy_(s.view(torch.int32))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, self.in_features)
        q, s = quantize_activation(x2, self.group)
        return self.matmul_quantized(q, s, x.dtype).reshape(*x.shape[:-1], self.out_features)

    def matmul_quantized(self, q: torch.Tensor, s: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        """This layer on rows already rotated and quantized with its group, as ``[M, N]``:
        one tcgen05 GEMM with the rescale and bias in its epilogue."""
        return kernels.gemm_w8a8(q, self.weight, s, self.scale, self.bias, dtype)

    def extra_repr(self) -> str:
        return f"in_features={self.in_features}, out_features={self.out_features}, group={self.group}"


class Int8Embedding(nn.Module):
    """``nn.Embedding`` over an int8 ConvRot table with one fp32 scale per row
    (_int8.py:173-197): a lookup gathers, rescales and un-rotates only the requested rows."""

    def __init__(self, num_embeddings: int, embedding_dim: int, group: int = GROUP, device=None):
        super().__init__()
        if group and embedding_dim % group:
            raise ValueError(f"embedding_dim {embedding_dim} is not a multiple of the ConvRot group {group}")
        self.num_embeddings, self.embedding_dim, self.group = num_embeddings, embedding_dim, group
        self.out_dtype = torch.float32
        self.register_buffer("weight", torch.empty(num_embeddings, embedding_dim, dtype=torch.int8, device=device))
        self.register_buffer("scale_bits", torch.empty(num_embeddings, dtype=torch.int32, device=device))

    @property
    def scale(self) -> torch.Tensor:
        return self.scale_bits.view(torch.float32)

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        flat = ids.reshape(-1)
        rows = dequantize_weight(self.weight[flat], self.scale[flat], self.group)
        return rows.reshape(*ids.shape, self.embedding_dim).to(self.out_dtype)

    def extra_repr(self) -> str:
        return f"{self.num_embeddings}, {self.embedding_dim}, group={self.group}"


def int8_mlp(x: torch.Tensor, l1: Int8Linear, l2: Int8Linear) -> torch.Tensor:
    """``l2(gelu(l1(x)))`` with erf-GELU (_int8.py:326-345): quantize x, GEMM 1 with rescale,
    bias and GELU (rounded to x's dtype) in its epilogue, quantize, GEMM 2."""
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("int8_mlp runs on fp16 / bf16 activations")
    x2 = x.reshape(-1, l1.in_features)
    q, s = quantize_activation(x2, l1.group)
    h = kernels.gemm_w8a8(q, l1.weight, s, l1.scale, l1.bias, x.dtype, gelu=_lib.GELU_ERF)
    q2, s2 = quantize_activation(h, l2.group)
    return l2.matmul_quantized(q2, s2, x.dtype).reshape(*x.shape[:-1], l2.out_features)


def _gelu_quantize(h: torch.Tensor, group: int):
    """:func:`quantize_activation` of ``gelu(h)`` rounded to ``h.dtype`` in one row pass
    (_int8.py:348-358)."""
    return kernels.quant_rows(h, group, _lib.GELU_ERF)


# ─── checkpoint plumbing (_int8.py:446-520) ─────────────────────────────────────────────

def _parent(model: nn.Module, name: str):
    head, _, leaf = name.rpartition(".")
    return (model.get_submodule(head) if head else model), leaf


def int8_layers(state_dict: dict) -> dict[str, int]:
    """``{layer: ConvRot group (0 = none)}`` for every ``comfy_quant``-tagged layer of a ComfyUI
    quantized checkpoint; empty for a plain one. Formats other than int8_tensorwise raise."""
    found = {}
    suffix = ".comfy_quant"
    for key, tag in state_dict.items():
        if not key.endswith(suffix):
            continue
        layer = key[: -len(suffix)]
        meta = json.loads(bytes(tag.tolist()).decode())
        fmt = meta.get("format")
        if fmt != "int8_tensorwise":
            raise ValueError(f"{layer}: quantized format {fmt!r} is not supported "
                             f"(diffucore_b200 reads int8_tensorwise only)")
        found[layer] = int(meta.get("convrot_groupsize", 256)) if meta.get("convrot") else 0
    return found


def adopt_int8_layers(model: nn.Module, state_dict: dict, layers: dict[str, int]) -> dict:
    """Swap each tagged ``nn.Linear`` of a meta-built ``model`` for an :class:`Int8Linear` and
    rename its checkpoint entries (``weight_scale`` -> ``scale_bits``) so a strict
    ``load_state_dict`` follows."""
    for name, group in layers.items():
        parent, leaf = _parent(model, name)
        lin = getattr(parent, leaf)
        setattr(parent, leaf, Int8Linear(lin.in_features, lin.out_features, lin.bias is not None, group,
                                         device="meta"))
        scale = state_dict.pop(name + ".weight_scale").float().reshape(-1)
        state_dict[name + ".scale_bits"] = scale.expand(lin.out_features).contiguous().view(torch.int32)
        del state_dict[name + ".comfy_quant"]
    return state_dict


def adopt_int8_embedding(model: nn.Module, state_dict: dict, name: str, group: int) -> dict:
    """:func:`adopt_int8_layers` for an ``nn.Embedding``."""
    parent, leaf = _parent(model, name)
    emb = getattr(parent, leaf)
    setattr(parent, leaf, Int8Embedding(emb.num_embeddings, emb.embedding_dim, group, device="meta"))
    scale = state_dict.pop(name + ".weight_scale").float().reshape(-1)
    state_dict[name + ".scale_bits"] = scale.expand(emb.num_embeddings).contiguous().view(torch.int32)
    del state_dict[name + ".comfy_quant"]
    return state_dict


def quantize_linears(model: nn.Module, names, device, group: int = GROUP) -> int:
    """Replace the named ``nn.Linear`` layers with ConvRot :class:`Int8Linear` (quantized on
    ``device``, then moved back to the layer's own device)."""
    count = 0
    for name in names:
        parent, leaf = _parent(model, name)
        lin = getattr(parent, leaf)
        setattr(parent, leaf, Int8Linear.from_linear(lin, group, device).to(lin.weight.device))
        count += 1
    return count


def dequantize_linears(model: nn.Module, dtype: torch.dtype, device=None) -> int:
    """Turn every :class:`Int8Linear` back into an fp ``nn.Linear`` (working on ``device``)."""
    names = [n for n, m in model.named_modules() if isinstance(m, Int8Linear)]
    for name in names:
        parent, leaf = _parent(model, name)
        layer = getattr(parent, leaf)
        home = layer.weight.device
        work = layer.to(device) if device is not None else layer
        setattr(parent, leaf, work.to_linear(dtype).to(home))
    return len(names)


def lora_seed(name: str, path: str) -> int:
    """Deterministic stochastic-rounding seed per (layer, LoRA file)."""
    return zlib.crc32(f"{name}|{path}".encode())
