"""diffucore_b200: the quantized hot path of diffucore (W8A8 linear, activation quantizer,
INT8 flash attention) as hand-written sm_100a kernels behind a C-ABI, with diffucore's module
and operator API on top (``diffucore_b200._int8``, ``diffucore_b200._attention``)."""

from . import _lib
from ._attention import attention_bhld, attention_blhd, resolve_attention_backend, set_attention_backend
from ._int8 import Int8Linear, int8_mlp, quantize_activation

__all__ = ["Int8Linear", "int8_mlp", "quantize_activation", "attention_blhd", "attention_bhld",
           "resolve_attention_backend", "set_attention_backend"]
__version__ = "0.1.0"
