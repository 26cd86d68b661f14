"""B200 (sm_100a) scaled-dot-product-attention engine with gguf_train's attention API.

    from gguf_train_b200 import functional as F, MultiheadAttention
    out = F.scaled_dot_product_attention(q, k, v, is_causal=True)     # torch CUDA tensors

The kernels live in the native library gguf_train_b200/_lib/libgt_attn_b200.so (C ABI:
include/gtb_attn.h, include/gguf_train_attn.h). Importing this package loads it; a missing library
is an ImportError, never a silent fallback.
"""

from . import _C
from . import functional
from . import gguf_io
from . import handles
from .functional import (FlashAttentionFn, RoPEFn, decode_q8_0, dequantize_q8_0, q8_0_append, quantize_q8_0, rope,
                         scaled_dot_product_attention, sdpa_from_host)
from .modules import MultiheadAttention

__all__ = [
    "_C",
    "functional",
    "gguf_io",
    "handles",
    "FlashAttentionFn",
    "MultiheadAttention",
    "scaled_dot_product_attention",
    "sdpa_from_host",
    "quantize_q8_0",
    "q8_0_append",
    "rope",
    "RoPEFn",
    "dequantize_q8_0",
    "decode_q8_0",
]
