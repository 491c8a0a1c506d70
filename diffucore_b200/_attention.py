"""Attention dispatch with the B200 INT8 backend: the API of diffucore's
``diffucore.models._attention`` (src/diffucore/models/_attention.py) with its ``"int8_turing"``
branch served by this package's tcgen05 kernel.

The policy value stays ``"int8_turing"`` so pipelines and loaders are unchanged. Differences
from the reference, all widenings: fp16 **and** bf16 inputs, head dims 64 and 128, and a choice of
quantization mode (``"ref"``: the reference's per-token Q / mean-centred per-64-key K, the
default; ``"block64"``: per-64-token Q and K). The per-call eligibility guard keeps the
reference's meaning: inputs the INT8 kernel does not take (CPU tensors, fp32, other head dims,
unaligned strides) run exact SDPA, as they do in the reference. An eligible call whose native
library cannot load raises instead of silently running SDPA. The FA2-Turing backend is an sm75
package and never available here.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from . import _lib, kernels

_CHOICES = ("sdpa", "auto", "fa2_turing", "int8_turing")
_MODES = {"ref": _lib.MODE_REF, "block64": _lib.MODE_BLOCK64}
_int8_mode = "ref"


def set_int8_quant_mode(mode: str) -> None:
    """Process-wide default quantization mode of the INT8 backend: ``"ref"`` or ``"block64"``."""
    global _int8_mode
    if mode not in _MODES:
        raise ValueError(f"unknown INT8 attention mode {mode!r}; choose from {sorted(_MODES)}")
    _int8_mode = mode


def get_int8_quant_mode() -> str:
    return _int8_mode


def fa2_turing_available(device=None) -> bool:
    """FA2-Turing is an sm75-only extension (_attention.py:56-63); never usable on sm_100."""
    return False


def _int8_arch(device=None) -> str | None:
    """The arch the INT8 kernel is built for here: "100a" on sm_100, else None."""
    if not torch.cuda.is_available():
        return None
    return "100a" if torch.cuda.get_device_capability(device) == (10, 0) else None


def _library_error() -> str:
    try:
        _lib.load()
        return ""
    except _lib.NativeLibraryError as e:
        return str(e)


def int8_turing_available(device=None) -> bool:
    """Whether the INT8 kernel can run here: an sm_100 device and the prebuilt library
    (reference: _attention.py:81-86)."""
    if device is not None and getattr(torch.device(device), "type", None) == "cpu":
        return False
    return _int8_arch(device) is not None and not _library_error()


def _int8_requirements(policy):
    """(message, satisfied) pairs for running the INT8 kernel under ``policy``."""
    dev = torch.device(policy.device)
    yield "device is not CUDA", dev.type == "cuda"
    yield "GPU is not sm_100 (the INT8 kernels are built for sm_100a only)", (
        dev.type == "cuda" and _int8_arch(dev) is not None)
    yield "compute dtype is not fp16 or bf16", policy.compute_dtype in (torch.float16, torch.bfloat16)
    yield "incompatible with compile=True (the custom op graph-breaks in every block)", not getattr(
        policy, "compile", False)
    err = _library_error()
    yield f"INT8 kernel library unavailable: {err}", not err


def _fa2_requirements(policy):
    """(message, satisfied) pairs for FA2-Turing under ``policy`` (_attention.py:117-121): its
    package is sm75-only and not part of this build, so the first never holds; the rest are
    listed as the reference lists them, so an explicit request names every unmet one."""
    dev = torch.device(policy.device)
    yield "flash_attn_turing is not installed (an sm75-only package, not part of the B200 build)", False
    yield "device is not CUDA", dev.type == "cuda"
    yield "GPU is not Turing; the kernel is compiled for sm_75 only", (
        dev.type == "cuda" and torch.cuda.is_available() and torch.cuda.get_device_capability(dev) == (7, 5))
    yield "compute dtype is not fp16", policy.compute_dtype == torch.float16
    yield "incompatible with compile=True (the custom op graph-breaks in every block)", not getattr(
        policy, "compile", False)


def resolve_attention_backend(policy) -> str:
    """``"sdpa"`` as is; ``"auto"`` -> ``"sdpa"`` (FA2-Turing never applies on sm_100); an
    explicit ``"fa2_turing"`` / ``"int8_turing"`` raises on the first unmet requirement, so an
    A/B never silently runs the same backend twice (_attention.py:136-158)."""
    choice = policy.attention
    if choice not in _CHOICES:
        raise ValueError(f"policy.attention={choice!r}; choose from {_CHOICES}")
    if choice == "sdpa" or choice == "auto":
        return "sdpa"
    if choice == "int8_turing":
        failures = [msg for msg, ok in _int8_requirements(policy) if not ok]
        if failures:
            raise ValueError("policy.attention='int8_turing' can't run: " + "; ".join(failures))
        return "int8_turing"
    failures = [msg for msg, ok in _fa2_requirements(policy) if not ok]
    raise ValueError("policy.attention='fa2_turing' can't run: " + "; ".join(failures))


def set_attention_backend(module: torch.nn.Module, backend: str) -> int:
    """Stamp ``backend`` on every submodule with an ``attn_backend`` slot; ``int8_turing`` goes
    on self-attention only, modules with ``is_selfattn = False`` get SDPA (_attention.py:161-175).
    Returns the number stamped."""
    n = 0
    for m in module.modules():
        if hasattr(m, "attn_backend"):
            cross = not getattr(m, "is_selfattn", True)
            m.attn_backend = "sdpa" if backend == "int8_turing" and cross else backend
            n += 1
    return n


def _int8_eligible(*ts: torch.Tensor) -> bool:
    """Per-call guard (_attention.py:184-192, widened to bf16 and D = 64): CUDA, one 16-bit dtype,
    head dim 64 or 128 and packed, other strides multiples of 8, 16-byte aligned."""
    if not ts or ts[0].dtype not in (torch.float16, torch.bfloat16):
        return False
    dtype = ts[0].dtype
    return all(
        t.is_cuda and t.dtype == dtype and t.dim() == 4 and t.shape[-1] in (64, 128)
        and t.stride(-1) == 1 and all(s % 8 == 0 for s in t.stride()[:-1])
        and t.data_ptr() % 16 == 0
        for t in ts
    ) and _int8_arch(ts[0].device) is not None


def _run_int8(q, k, v, mode):
    m = _MODES[mode if mode is not None else _int8_mode]
    return kernels.attn_int8(q, k, v, q.shape[-1] ** -0.5, m)


def _sdpa_blhd(q, k, v):
    out = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    return out.transpose(1, 2)


def attention_blhd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, backend: str = "sdpa",
                   null_keys: int = 0, quant_mode: str | None = None) -> torch.Tensor:
    """Attention over ``(B, L, H, D)`` q/k/v -> ``(B, Lq, H*D)`` (_attention.py:195-227).
    ``null_keys`` counts all-zero key/value rows left off ``k``/``v``; they are padded back on."""
    B, Lq = q.shape[0], q.shape[1]
    if null_keys:
        k = F.pad(k, (0, 0, 0, 0, 0, null_keys))
        v = F.pad(v, (0, 0, 0, 0, 0, null_keys))
    if backend == "int8_turing" and _int8_eligible(q, k, v):
        return _run_int8(q, k, v, quant_mode).reshape(B, Lq, -1)
    return _sdpa_blhd(q, k, v).reshape(B, Lq, -1)


def attention_bhld(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, backend: str = "sdpa",
                   quant_mode: str | None = None) -> torch.Tensor:
    """Attention over ``(B, H, L, D)`` q/k/v -> ``(B, Lq, H*D)`` (FLUX layout, post-RoPE,
    _attention.py:261-279). The INT8 kernel reads the transposed views in place."""
    B, Lq = q.shape[0], q.shape[2]
    if backend == "int8_turing":
        qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
        if _int8_eligible(qt, kt, vt):
            return _run_int8(qt, kt, vt, quant_mode).reshape(B, Lq, -1)
    out = F.scaled_dot_product_attention(q, k, v)
    return out.transpose(1, 2).reshape(B, Lq, -1)
