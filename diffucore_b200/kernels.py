"""Torch-tensor front of the C-ABI: allocates outputs and workspaces with the caching
allocator, passes raw pointers and the current stream, raises on a non-zero status.

These are the only entry points the module layer (``_int8``, ``_attention``) uses. They run
on sm_100 CUDA tensors only and raise for anything else; there is no CPU implementation.
"""

from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

_DTYPE = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise RuntimeError("diffucore_b200 kernels run on CUDA tensors only (got a "
                               f"{t.device.type} tensor); there is no CPU path")


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p:
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


def quant_rows(x2: torch.Tensor, group: int = 0, gelu: int = _lib.GELU_NONE):
    """``(int8 [M, K], fp32 [M])`` per-row codes and scales of ``x2`` [M, K] (any row stride)."""
    _require_cuda(x2)
    if x2.dim() != 2:
        raise ValueError("quant_rows expects a 2-D tensor")
    if x2.dtype not in _DTYPE:
        raise TypeError(f"quant_rows: unsupported dtype {x2.dtype}")
    if x2.stride(1) != 1:
        x2 = x2.contiguous()
    M, K = x2.shape
    q = torch.empty(M, K, device=x2.device, dtype=torch.int8)
    s = torch.empty(M, device=x2.device, dtype=torch.float32)
    lib = _lib.load()
    with torch.cuda.device(x2.device):
        _lib.check(lib.dc_quant_rows(_ptr(x2), _DTYPE[x2.dtype], M, K, x2.stride(0), int(group), int(gelu),
                                     _ptr(q), _ptr(s), _stream(x2)))
    return q, s


def _gemm_operand(t: torch.Tensor) -> torch.Tensor:
    if t.dtype != torch.int8 or t.dim() != 2:
        raise TypeError("GEMM operands are 2-D int8")
    if t.stride(1) != 1 or t.stride(0) % 16 or t.data_ptr() % 16:
        t = t.contiguous()
    return t


def _pad_k(q: torch.Tensor, w: torch.Tensor):
    """Zero-pad K to a multiple of 16 (the TMA row pitch); zeros add nothing to the dot products."""
    K = q.shape[1]
    if K % 16 == 0:
        return q, w
    pad = 16 - K % 16
    return torch.nn.functional.pad(q, (0, pad)), torch.nn.functional.pad(w, (0, pad))


def gemm_w8a8(q: torch.Tensor, w: torch.Tensor, sx: torch.Tensor | None, sw: torch.Tensor | None,
              bias: torch.Tensor | None = None, out_dtype: torch.dtype = torch.bfloat16,
              gelu: int = _lib.GELU_NONE) -> torch.Tensor:
    """``epilogue(q @ w.T)``: int32 (``out_dtype=torch.int32``) or rescaled + bias in bf16/fp16."""
    _require_cuda(q, w)
    if q.shape[1] != w.shape[1]:
        raise ValueError(f"K mismatch: q {tuple(q.shape)} vs w {tuple(w.shape)}")
    q, w = _pad_k(_gemm_operand(q), _gemm_operand(w))
    M, K = q.shape
    N = w.shape[0]
    if out_dtype == torch.int32:
        code = _lib.DTYPE_I32
        sx = sw = None
    elif out_dtype in (torch.bfloat16, torch.float16):
        code = _DTYPE[out_dtype]
        sx = sx.to(torch.float32).contiguous()
        sw = sw.to(torch.float32).contiguous()
        if bias is not None:
            bias = bias.to(out_dtype).contiguous()
    else:
        raise TypeError(f"gemm_w8a8: unsupported output dtype {out_dtype}")
    out = torch.empty(M, N, device=q.device, dtype=out_dtype)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        _lib.check(lib.dc_gemm_w8a8(_ptr(q), q.stride(0), _ptr(w), w.stride(0), _ptr(sx), _ptr(sw), _ptr(bias),
                                    _ptr(out), out.stride(0), code, M, N, K, int(gelu), _stream(q)))
    return out


def rescale(acc: torch.Tensor, sx: torch.Tensor, sw: torch.Tensor, bias: torch.Tensor | None,
            dtype: torch.dtype) -> torch.Tensor:
    """``dtype(acc * (sx[:, None] * sw)) (+ bias in dtype)`` for an int32 ``acc`` [M, N]."""
    _require_cuda(acc)
    if acc.dtype != torch.int32 or acc.dim() != 2:
        raise TypeError("rescale expects a 2-D int32 accumulator")
    if dtype not in (torch.bfloat16, torch.float16):
        raise TypeError(f"rescale: unsupported dtype {dtype}")
    acc = acc if acc.stride(1) == 1 else acc.contiguous()
    M, N = acc.shape
    sx = sx.to(torch.float32).contiguous()
    sw = sw.to(torch.float32).contiguous()
    if bias is not None:
        bias = bias.to(dtype).contiguous()
    out = torch.empty(M, N, device=acc.device, dtype=dtype)
    lib = _lib.load()
    with torch.cuda.device(acc.device):
        _lib.check(lib.dc_rescale(_ptr(acc), acc.stride(0), _ptr(sx), _ptr(sw), _ptr(bias), _ptr(out),
                                  out.stride(0), _DTYPE[dtype], M, N, _stream(acc)))
    return out


def gemm_w8a8_into(q: torch.Tensor, w: torch.Tensor, sx: torch.Tensor, sw: torch.Tensor,
                   bias: torch.Tensor | None, out: torch.Tensor, *, ldo: int | None = None,
                   gelu: int = _lib.GELU_NONE, gate: torch.Tensor | None = None,
                   residual: torch.Tensor | None = None, col_block: int = 0, block_stride: int = 0) -> None:
    """``gemm_w8a8`` into caller memory, with the DiT epilogue options of ``dc_gemm_w8a8_ex``.

    ``out`` supplies the base address and dtype; rows are ``ldo`` elements apart (default
    ``out.stride(0)``). ``gate``/``residual`` (residual a row-strided [M, N] view, possibly ``out``
    itself) give ``out = dtype(residual + dtype(gate * y))``. ``col_block > 0`` writes the
    [N / col_block, M, col_block] block layout with blocks ``block_stride`` elements apart.
    Operands are used as given (no copies): q [M, K] and w [N, K] int8 with 16-byte aligned rows,
    sx [M], sw [N] fp32, bias and gate [N] in ``out``'s dtype, all contiguous."""
    _require_cuda(q, w, out)
    M, K = q.shape
    N = w.shape[0]
    if ldo is None:
        ldo = out.stride(0)
    ldr = residual.stride(0) if residual is not None else 0
    lib = _lib.load()
    _lib.check(lib.dc_gemm_w8a8_ex(_ptr(q), q.stride(0), _ptr(w), w.stride(0), _ptr(sx), _ptr(sw), _ptr(bias),
                                   int(gelu), _ptr(gate), _ptr(residual), ldr, _ptr(out), int(ldo), int(col_block),
                                   int(block_stride), _DTYPE[out.dtype], M, N, K, _stream(q)))


def ln_mod_quant(x: torch.Tensor, shift: torch.Tensor, scale: torch.Tensor, group: int,
                 q: torch.Tensor | None = None, s: torch.Tensor | None = None):
    """Codes of ``dtype(dtype(dtype(1 + scale) * LN(x)) + shift)`` per row of ``x`` [M, K]
    (LayerNorm without affine, eps 1e-6), as ``dc_quant_rows`` would give for that activation.
    ``shift``/``scale`` are [K] vectors in x's dtype. Returns ``(q int8 [M, K], s fp32 [M])``."""
    _require_cuda(x)
    M, K = x.shape
    if q is None:
        q = torch.empty(M, K, device=x.device, dtype=torch.int8)
    if s is None:
        s = torch.empty(M, device=x.device, dtype=torch.float32)
    lib = _lib.load()
    _lib.check(lib.dc_ln_mod_quant(_ptr(x), _DTYPE[x.dtype], M, K, x.stride(0), _ptr(shift), _ptr(scale), max(M, 1),
                                   0, int(group), _ptr(q), _ptr(s), _stream(x)))
    return q, s


def quant_rows_into(x: torch.Tensor, group: int, q: torch.Tensor, s: torch.Tensor) -> None:
    """``quant_rows`` of a row-strided [M, K] view into caller buffers (q [M, K] contiguous)."""
    _require_cuda(x)
    M, K = x.shape
    lib = _lib.load()
    _lib.check(lib.dc_quant_rows(_ptr(x), _DTYPE[x.dtype], M, K, x.stride(0), int(group), _lib.GELU_NONE,
                                 _ptr(q), _ptr(s), _stream(x)))


def quant_rows_seg(recv: torch.Tensor, x2: torch.Tensor | None, group: int, q: torch.Tensor,
                   s: torch.Tensor) -> None:
    """Codes of the rows ``cat([recv[0], ..., recv[P-1], x2], dim=1)`` for an all-to-all receive
    buffer ``recv`` [P, M, W] (contiguous) and an optional row-strided ``x2`` [M, K2], without
    forming the concatenation."""
    _require_cuda(recv)
    P, M, W = recv.shape
    K = P * W + (x2.shape[1] if x2 is not None else 0)
    lib = _lib.load()
    _lib.check(lib.dc_quant_rows_seg(_ptr(recv), _DTYPE[recv.dtype], M, K, W, W, M * W, P * W, _ptr(x2),
                                     x2.stride(0) if x2 is not None else 0, int(group), _ptr(q), _ptr(s),
                                     _stream(recv)))


def qk_norm_rope(qkv: torch.Tensor, q_scale0: torch.Tensor, k_scale0: torch.Tensor, pe: torch.Tensor,
                 q_scale1: torch.Tensor | None = None, k_scale1: torch.Tensor | None = None,
                 split_row: int | None = None, q8_workspace: torch.Tensor | None = None,
                 write_q: bool = True) -> None:
    """In place on ``qkv`` [L, 3, H, 128] (row-strided): RMSNorm of q and k per head with their
    scales, then RoPE with ``pe`` [L, 64, 2, 2] fp32. Rows below ``split_row`` use the ``*0``
    scales, the rest the ``*1`` scales. With ``q8_workspace`` (an attention workspace for
    (1, H, L, L, 128) in the reference quant mode) the Q codes and scales go straight into it
    (``dc_qk_norm_rope_q8``); :func:`attn_int8` with ``q_ready=True`` then quantizes only K, and
    ``write_q=False`` leaves q in ``qkv`` untouched."""
    _require_cuda(qkv, pe)
    L, three, H, D = qkv.shape
    if three != 3 or qkv.stride(3) != 1 or qkv.stride(2) != D or qkv.stride(1) != H * D:
        raise ValueError("qk_norm_rope expects rows laid out as [3, H, D]")
    if split_row is None:
        split_row = L
    for sc in (q_scale0, k_scale0, q_scale1, k_scale1):
        if sc is not None and (sc.dtype != qkv.dtype or sc.numel() != D or not sc.is_contiguous()):
            raise ValueError(f"qk_norm_rope: scales must be contiguous [{D}] tensors in {qkv.dtype}")
    if pe.dtype != torch.float32 or not pe.is_contiguous() or pe.numel() < L * D * 2:
        raise ValueError(f"qk_norm_rope: pe must be a contiguous fp32 table of at least [{L}, {D // 2}, 2, 2]")
    lib = _lib.load()
    if q8_workspace is None:
        _lib.check(lib.dc_qk_norm_rope(_ptr(qkv), _DTYPE[qkv.dtype], L, H, D, qkv.stride(0), 0, H * D,
                                       _ptr(q_scale0), _ptr(k_scale0), _ptr(q_scale1), _ptr(k_scale1),
                                       int(split_row), _ptr(pe), 0, _stream(qkv)))
        return
    lay = attn_workspace_layout(1, H, L, L, D, _lib.MODE_REF)
    if q8_workspace.numel() < lay["total"] or q8_workspace.dtype != torch.uint8:
        raise ValueError(f"qk_norm_rope: q8_workspace needs {lay['total']} bytes (uint8)")
    base = q8_workspace.data_ptr()
    _lib.check(lib.dc_qk_norm_rope_q8(_ptr(qkv), _DTYPE[qkv.dtype], L, H, D, qkv.stride(0), 0, H * D,
                                      _ptr(q_scale0), _ptr(k_scale0), _ptr(q_scale1), _ptr(k_scale1),
                                      int(split_row), _ptr(pe), 0, ctypes.c_void_p(base + lay["q_codes"]),
                                      ctypes.c_void_p(base + lay["q_scale"]), lay["Lq_pad"], int(bool(write_q)),
                                      _stream(qkv)))


def attn_workspace_layout(B: int, H: int, Lq: int, Lk: int, D: int, mode: int) -> dict:
    lay = (ctypes.c_int64 * 8)()
    _lib.check(_lib.load().dc_attn_workspace_layout(B, H, Lq, Lk, D, mode, lay))
    keys = ("Lq_pad", "Lk_pad", "q_codes", "k_codes", "q_scale", "k_scale", "ksum", "total")
    return dict(zip(keys, (int(v) for v in lay)))


def _blhd_strides(t: torch.Tensor):
    return _lib.i64_array((t.stride(0), t.stride(1), t.stride(2)))


def _check_attn_inputs(q, k, v):
    _require_cuda(q, k, v)
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t.dim() != 4 or t.stride(3) != 1:
            raise ValueError(f"{name} must be (B, L, H, D) with a contiguous head dim")
    if not (q.dtype == k.dtype == v.dtype) or q.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError("q, k, v must share one dtype, fp16 or bf16")
    B, Lq, H, D = q.shape
    Lk = k.shape[1]
    if k.shape != (B, Lk, H, D) or v.shape != (B, Lk, H, D):
        raise ValueError(f"q, k, v shapes disagree: {tuple(q.shape)}, {tuple(k.shape)}, {tuple(v.shape)}")
    return B, Lq, Lk, H, D


def attn_int8(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float,
              mode: int = _lib.MODE_REF, workspace: torch.Tensor | None = None,
              out: torch.Tensor | None = None, q_ready: bool = False) -> torch.Tensor:
    """INT8 attention over ``(B, L, H, D)`` q/k/v (any strides with stride(-1) == 1 and the
    others multiples of 8) -> contiguous ``(B, Lq, H, D)`` in the input dtype. Shapes whose grid
    fills the GPU poorly (few heads over long sequences, a sequence-parallel rank's share) run
    :func:`attn_int8_split` with the key-range count :func:`choose_attn_split` picks; the
    environment variable ``DC_ATTN_SPLIT=0`` turns that routing off. ``q_ready``: ``workspace``
    already holds the Q codes and scales (:func:`qk_norm_rope` with ``q8_workspace``), so only K
    is quantized here and ``q`` is not read."""
    B, Lq, Lk, H, D = _check_attn_inputs(q, k, v)
    if q_ready and workspace is None:
        raise ValueError("attn_int8: q_ready needs the workspace that holds the Q codes")
    if os.environ.get("DC_ATTN_SPLIT", "auto") != "0":
        nsplit = choose_attn_split(B, H, Lq, Lk, _sm_count(q.device), D=D)
        if nsplit > 1:
            return attn_int8_split(q, k, v, sm_scale, nsplit, mode, workspace=workspace, out=out, q_ready=q_ready)
    lib = _lib.load()
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.dc_attn_workspace_size(B, H, Lq, Lk, D, int(mode), ctypes.byref(nbytes)))
    if workspace is None or workspace.numel() < nbytes.value:
        if q_ready:
            raise ValueError(f"attn_int8: workspace below the {nbytes.value} bytes this shape needs")
        workspace = torch.empty(nbytes.value, device=q.device, dtype=torch.uint8)
    if out is None:
        out = torch.empty(B, Lq, H, D, device=q.device, dtype=q.dtype)
    with torch.cuda.device(q.device):
        if q_ready:
            _lib.check(lib.dc_attn_int8_prep_k(_ptr(k), _DTYPE[k.dtype], B, H, Lq, Lk, D, _blhd_strides(k), int(mode),
                                               _ptr(workspace), workspace.numel(), _stream(k)))
            _lib.check(lib.dc_attn_int8_main(_ptr(v), _DTYPE[v.dtype], B, H, Lq, Lk, D, _blhd_strides(v),
                                             float(sm_scale), int(mode), _ptr(out), _blhd_strides(out),
                                             _ptr(workspace), workspace.numel(), _stream(v)))
        else:
            _lib.check(lib.dc_attn_int8_fwd(_ptr(q), _ptr(k), _ptr(v), _DTYPE[q.dtype], B, H, Lq, Lk, D,
                                            _blhd_strides(q), _blhd_strides(k), _blhd_strides(v),
                                            float(sm_scale), int(mode), _ptr(out), _blhd_strides(out),
                                            _ptr(workspace), workspace.numel(), _stream(q)))
    return out


_SMS: dict = {}


def _sm_count(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SMS[idx]


def choose_attn_split(B: int, H: int, Lq: int, Lk: int, sms: int = 148, max_split: int = 4, D: int = 128) -> int:
    """Key ranges for :func:`attn_int8_split` (1 = do not split), from a wave-count model in units
    of one two-tile CTA's 128-key step (~2.4 us on a B200): the two-tile kernel runs
    ceil(Lq / 256) CTAs per head, each for its key tiles plus about one tile's worth of prologue
    and epilogue; the single-tile kernel the unsplit call would otherwise choose takes 0.61 of a
    two-tile CTA's time for 128 rows. A split also pays for its combine pass: about 1.3 units of
    launch and tail plus the fp32 partials written and read back (ranges x 2 x B H Lq D x 4 bytes,
    ~14 MB per unit at HBM speed). A split is chosen only when it saves at least 10 % against the
    better unsplit kernel. Measured on a B200 (3 heads, mode ref): 16896 tokens split in two
    0.486 ms against 0.529 unsplit; 4608 tokens 0.076 against 0.071, so not split."""
    qctas = B * H * -(-Lq // 256)
    n = -(-Lk // 128)

    def waves(ctas: int) -> int:
        return -(-ctas // sms)

    def cost_split(r: int) -> float:
        tps = -(-n // r)
        ranges = -(-n // tps)
        cost = waves(qctas * ranges) * (tps + 1)
        if ranges > 1:
            cost += 1.3 + ranges * 2 * B * H * Lq * D * 4 / 14e6
        return cost

    unsplit = min(cost_split(1), 0.61 * waves(2 * qctas) * (n + 1))
    best = min(range(1, min(max_split, n) + 1), key=lambda r: (cost_split(r), r))
    return best if best > 1 and cost_split(best) < 0.9 * unsplit else 1


def attn_split_partials_bytes(B: int, H: int, Lq: int, Lk: int, D: int, nsplit: int) -> int:
    nbytes = ctypes.c_size_t(0)
    _lib.check(_lib.load().dc_attn_split_partials_size(B, H, Lq, Lk, D, int(nsplit), ctypes.byref(nbytes)))
    return int(nbytes.value)


def attn_int8_split(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, sm_scale: float, nsplit: int,
                    mode: int = _lib.MODE_REF, workspace: torch.Tensor | None = None,
                    partials: torch.Tensor | None = None, out: torch.Tensor | None = None,
                    q_ready: bool = False) -> torch.Tensor:
    """:func:`attn_int8` with the keys divided into ``nsplit`` ranges (one CTA per 256 query rows and
    key range, then a merge of the ranges): the same result to rounding, for grids of few heads."""
    B, Lq, Lk, H, D = _check_attn_inputs(q, k, v)
    lib = _lib.load()
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.dc_attn_workspace_size(B, H, Lq, Lk, D, int(mode), ctypes.byref(nbytes)))
    if workspace is None or workspace.numel() < nbytes.value:
        if q_ready:
            raise ValueError(f"attn_int8_split: workspace below the {nbytes.value} bytes this shape needs")
        workspace = torch.empty(nbytes.value, device=q.device, dtype=torch.uint8)
    pbytes = attn_split_partials_bytes(B, H, Lq, Lk, D, nsplit)
    if partials is None or partials.numel() < pbytes:
        partials = torch.empty(pbytes, device=q.device, dtype=torch.uint8)
    if out is None:
        out = torch.empty(B, Lq, H, D, device=q.device, dtype=q.dtype)
    with torch.cuda.device(q.device):
        if q_ready:
            _lib.check(lib.dc_attn_int8_prep_k(_ptr(k), _DTYPE[k.dtype], B, H, Lq, Lk, D, _blhd_strides(k), int(mode),
                                               _ptr(workspace), workspace.numel(), _stream(k)))
        else:
            _lib.check(lib.dc_attn_int8_prep(_ptr(q), _ptr(k), _DTYPE[q.dtype], B, H, Lq, Lk, D, _blhd_strides(q),
                                             _blhd_strides(k), int(mode), _ptr(workspace), workspace.numel(),
                                             _stream(q)))
        _lib.check(lib.dc_attn_int8_main_split(_ptr(v), _DTYPE[v.dtype], B, H, Lq, Lk, D, _blhd_strides(v),
                                               float(sm_scale), int(mode), _ptr(out), _blhd_strides(out),
                                               _ptr(workspace), workspace.numel(), int(nsplit), _ptr(partials),
                                               partials.numel(), _stream(v)))
    return out


def attn_int8_prep(q: torch.Tensor, k: torch.Tensor, mode: int = _lib.MODE_REF) -> dict:
    """The int8 codes and scales the attention computes for ``q``/``k`` (B, L, H, D):
    ``q_codes`` [B, H, Lq, D], ``q_scale`` [B, H, Lq], ``k_codes`` [B, H, Lk, D],
    ``k_scale`` [B, H, ceil(Lk / 64)] and, in mode REF, ``ksum`` [B, H, D]."""
    B, Lq, Lk, H, D = _check_attn_inputs(q, k, k)
    lay = attn_workspace_layout(B, H, Lq, Lk, D, int(mode))
    ws = torch.zeros(lay["total"], device=q.device, dtype=torch.uint8)
    lib = _lib.load()
    with torch.cuda.device(q.device):
        _lib.check(lib.dc_attn_int8_prep(_ptr(q), _ptr(k), _DTYPE[q.dtype], B, H, Lq, Lk, D, _blhd_strides(q),
                                         _blhd_strides(k), int(mode), _ptr(ws), ws.numel(), _stream(q)))
    Lqp, Lkp = lay["Lq_pad"], lay["Lk_pad"]
    BH = B * H

    def view(off, n, dtype, shape):
        item = torch.tensor([], dtype=dtype).element_size()
        return ws[off: off + n * item].view(dtype).view(*shape)

    res = {
        "q_codes": view(lay["q_codes"], BH * Lqp * D, torch.int8, (B, H, Lqp, D))[:, :, :Lq].clone(),
        "k_codes": view(lay["k_codes"], BH * Lkp * D, torch.int8, (B, H, Lkp, D))[:, :, :Lk].clone(),
        "q_scale": view(lay["q_scale"], BH * Lqp, torch.float32, (B, H, Lqp))[:, :, :Lq].clone(),
        "k_scale": view(lay["k_scale"], BH * (Lkp // 64), torch.float32, (B, H, Lkp // 64))[:, :, :(Lk + 63) // 64].clone(),
    }
    if mode == _lib.MODE_REF:
        res["ksum"] = view(lay["ksum"], BH * D, torch.float32, (B, H, D)).clone()
    return res


def selftest_wait_timeout(device: torch.device | str = "cuda", limit_cycles: int = 2_000_000) -> tuple[int, int]:
    """Run the bounded-wait self-test kernel; returns (kernel status, device error word)."""
    device = torch.device(device)
    status = torch.zeros(1, device=device, dtype=torch.int32)
    lib = _lib.load()
    with torch.cuda.device(device):
        _lib.device_error(clear=True)
        _lib.check(lib.dc_selftest_wait_timeout(int(limit_cycles), _ptr(status), _stream(status)))
        torch.cuda.synchronize(device)
        return int(status.item()), _lib.device_error(clear=True)


class AttnPlan:
    """A prepared INT8 attention call for fixed shapes: one workspace, reusable across calls.
    ``prep`` quantizes Q/K into the workspace, ``main`` runs the tensor-core kernel over it;
    ``__call__`` does both (the same work as :func:`attn_int8`)."""

    def __init__(self, B: int, H: int, Lq: int, Lk: int, D: int, dtype: torch.dtype, mode: int,
                 device: torch.device | str = "cuda"):
        self.B, self.H, self.Lq, self.Lk, self.D = B, H, Lq, Lk, D
        self.dtype, self.mode = dtype, int(mode)
        self.layout = attn_workspace_layout(B, H, Lq, Lk, D, self.mode)
        self.workspace = torch.empty(self.layout["total"], device=device, dtype=torch.uint8)

    def prep(self, q: torch.Tensor, k: torch.Tensor) -> None:
        lib = _lib.load()
        _lib.check(lib.dc_attn_int8_prep(_ptr(q), _ptr(k), _DTYPE[q.dtype], self.B, self.H, self.Lq, self.Lk,
                                         self.D, _blhd_strides(q), _blhd_strides(k), self.mode,
                                         _ptr(self.workspace), self.workspace.numel(), _stream(q)))

    def main(self, v: torch.Tensor, out: torch.Tensor, sm_scale: float) -> torch.Tensor:
        lib = _lib.load()
        _lib.check(lib.dc_attn_int8_main(_ptr(v), _DTYPE[v.dtype], self.B, self.H, self.Lq, self.Lk, self.D,
                                         _blhd_strides(v), float(sm_scale), self.mode, _ptr(out),
                                         _blhd_strides(out), _ptr(self.workspace), self.workspace.numel(),
                                         _stream(v)))
        return out

    def __call__(self, q, k, v, out, sm_scale):
        self.prep(q, k)
        return self.main(v, out, sm_scale)


def selftest_exp2(x: torch.Tensor):
    """(FMA-pipe exp2 used by the attention softmax, CUDA exp2f) of a CUDA fp32 tensor."""
    _require_cuda(x)
    x = x.contiguous().float()
    poly, ref = torch.empty_like(x), torch.empty_like(x)
    _lib.check(_lib.load().dc_selftest_exp2(_ptr(x), _ptr(poly), _ptr(ref), x.numel(), _stream(x)))
    return poly, ref
