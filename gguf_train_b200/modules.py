"""nn.MultiheadAttention of gguf_train over the engine's attention.

Same constructor, forward signature, layouts (batch_first, unbatched), mask rules and error
messages as the reference (gguf_train/nn/modules/transformer.py:21-191). With need_weights=False
attention runs through this package's scaled_dot_product_attention (the sm_100a path); with the
default need_weights=True the reference materialises the weights with explicit matmul + softmax
(:153-166), and so does this module, in torch. The in/out projections are plain torch linear
layers (library GEMMs).
"""

from __future__ import annotations

import torch
from torch import nn

from . import functional as F


class MultiheadAttention(nn.Module):
    def __init__(self, embed_dim: int, num_heads: int, dropout: float = 0.0, bias: bool = True,
                 add_bias_kv: bool = False, add_zero_attn: bool = False, kdim: int | None = None,
                 vdim: int | None = None, batch_first: bool = False, device=None, dtype=None) -> None:
        super().__init__()
        self.embed_dim = int(embed_dim)
        self.num_heads = int(num_heads)
        self.head_dim = self.embed_dim // self.num_heads
        assert self.head_dim * self.num_heads == self.embed_dim, "embed_dim must be divisible by num_heads"
        self.dropout = float(dropout)
        self.batch_first = bool(batch_first)
        self.kdim = self.embed_dim if kdim is None else int(kdim)
        self.vdim = self.embed_dim if vdim is None else int(vdim)
        dt = dtype or torch.get_default_dtype()
        self._qkv_same = self.kdim == self.embed_dim and self.vdim == self.embed_dim
        if self._qkv_same:
            self.in_proj_weight = nn.Parameter(torch.empty((3 * self.embed_dim, self.embed_dim), dtype=dt, device=device))
            self.register_parameter("q_proj_weight", None)
            self.register_parameter("k_proj_weight", None)
            self.register_parameter("v_proj_weight", None)
            nn.init.xavier_uniform_(self.in_proj_weight)
        else:
            self.register_parameter("in_proj_weight", None)
            self.q_proj_weight = nn.Parameter(torch.empty((self.embed_dim, self.embed_dim), dtype=dt, device=device))
            self.k_proj_weight = nn.Parameter(torch.empty((self.embed_dim, self.kdim), dtype=dt, device=device))
            self.v_proj_weight = nn.Parameter(torch.empty((self.embed_dim, self.vdim), dtype=dt, device=device))
            nn.init.xavier_uniform_(self.q_proj_weight)
            nn.init.xavier_uniform_(self.k_proj_weight)
            nn.init.xavier_uniform_(self.v_proj_weight)
        if bias:
            self.in_proj_bias = nn.Parameter(torch.zeros((3 * self.embed_dim,), dtype=dt, device=device))
        else:
            self.register_parameter("in_proj_bias", None)
        self.out_proj = nn.Linear(self.embed_dim, self.embed_dim, bias=bias, device=device, dtype=dt)

    def forward(self, query, key, value, key_padding_mask=None, need_weights: bool = True, attn_mask=None,
                average_attn_weights: bool = True, is_causal: bool = False):
        is_batched = query.ndim == 3
        if not is_batched:
            if query.ndim != 2 or key.ndim != 2 or value.ndim != 2:
                raise RuntimeError(
                    "MultiheadAttention: query, key and value must all be 3-D (batched) or all 2-D (unbatched), "
                    f"got {query.ndim}-D, {key.ndim}-D and {value.ndim}-D"
                )
            batch_dim = 0 if self.batch_first else 1
            query, key, value = query.unsqueeze(batch_dim), key.unsqueeze(batch_dim), value.unsqueeze(batch_dim)
            if key_padding_mask is not None:
                if key_padding_mask.ndim != 1:
                    raise RuntimeError(
                        "MultiheadAttention: key_padding_mask of an unbatched input must be 1-D (S), "
                        f"got {list(key_padding_mask.shape)}"
                    )
                key_padding_mask = key_padding_mask.unsqueeze(0)
        elif key.ndim != 3 or value.ndim != 3:
            raise RuntimeError(
                "MultiheadAttention: query, key and value must all be 3-D (batched) or all 2-D (unbatched), "
                f"got {query.ndim}-D, {key.ndim}-D and {value.ndim}-D"
            )
        if not self.batch_first:
            query, key, value = query.transpose(0, 1), key.transpose(0, 1), value.transpose(0, 1)
        B, L, E = query.shape
        S = key.shape[1]
        if self._qkv_same:
            wq, wk, wv = self.in_proj_weight.chunk(3, dim=0)
        else:
            wq, wk, wv = self.q_proj_weight, self.k_proj_weight, self.v_proj_weight
        if self.in_proj_bias is not None:
            bq, bk, bv = self.in_proj_bias.chunk(3, dim=0)
        else:
            bq = bk = bv = None
        q = torch.nn.functional.linear(query, wq, bq).reshape((B, L, self.num_heads, self.head_dim)).transpose(1, 2)
        k = torch.nn.functional.linear(key, wk, bk).reshape((B, S, self.num_heads, self.head_dim)).transpose(1, 2)
        v = torch.nn.functional.linear(value, wv, bv).reshape((B, S, self.num_heads, self.head_dim)).transpose(1, 2)

        mask = None
        if attn_mask is not None:
            if attn_mask.ndim == 2:
                if tuple(attn_mask.shape) != (L, S):
                    raise RuntimeError(f"MultiheadAttention: the 2D attn_mask has shape {list(attn_mask.shape)}, expected {[L, S]}")
                mask = self._additive_mask(attn_mask, q.dtype, "attn_mask").reshape((1, 1, L, S))
            elif attn_mask.ndim == 3:
                if tuple(attn_mask.shape) != (B * self.num_heads, L, S):
                    raise RuntimeError(
                        f"MultiheadAttention: the 3D attn_mask has shape {list(attn_mask.shape)}, "
                        f"expected {[B * self.num_heads, L, S]}"
                    )
                mask = self._additive_mask(attn_mask, q.dtype, "attn_mask").reshape((B, self.num_heads, L, S))
            else:
                raise RuntimeError(f"MultiheadAttention: attn_mask must be 2D or 3D, got {attn_mask.ndim}D")
        if key_padding_mask is not None:
            if tuple(key_padding_mask.shape) != (B, S):
                raise RuntimeError(
                    f"MultiheadAttention: key_padding_mask has shape {list(key_padding_mask.shape)}, expected {[B, S]}"
                )
            km = self._additive_mask(key_padding_mask, q.dtype, "key_padding_mask").reshape((B, 1, 1, S))
            mask = km if mask is None else (mask + km)

        scale = 1.0 / (self.head_dim ** 0.5)
        if not need_weights:
            attn_out = F.scaled_dot_product_attention(
                q, k, v, attn_mask=mask, dropout_p=self.dropout if self.training else 0.0, is_causal=is_causal,
                scale=scale,
            )
            attn_weights = None
        else:
            scores = q.matmul(k.transpose(-2, -1)) * scale
            if is_causal:
                cm = torch.ones((L, S), dtype=q.dtype, device=q.device).triu(diagonal=1) * (-1e9)
                scores = scores + cm
            if mask is not None:
                scores = scores + mask
            attn_weights = torch.softmax(scores, dim=-1)
            if self.dropout > 0.0 and self.training:
                attn_weights = torch.nn.functional.dropout(attn_weights, p=self.dropout, training=True)
            attn_out = attn_weights.matmul(v)
            if average_attn_weights:
                attn_weights = attn_weights.mean(dim=1)
        out = attn_out.transpose(1, 2).reshape((B, L, E))
        out = self.out_proj(out)
        if not self.batch_first:
            out = out.transpose(0, 1)
        if not is_batched:
            out = out.squeeze(1 if not self.batch_first else 0)
            if attn_weights is not None:
                attn_weights = attn_weights.squeeze(0)
        return out, attn_weights

    @staticmethod
    def _additive_mask(mask, dtype, name: str):
        """torch.nn convention (transformer.py:179-191): True in a bool attn_mask or key_padding_mask
        marks a position that must NOT be attended; it becomes -1e9. A float mask is added as is."""
        if mask.dtype == torch.bool:
            return torch.zeros(mask.shape, dtype=dtype, device=mask.device).masked_fill(mask, -1e9)
        if not mask.is_floating_point():
            raise RuntimeError(f"MultiheadAttention: {name} must be a boolean or floating point tensor, got {mask.dtype}")
        return mask if mask.dtype == dtype else mask.to(dtype)
