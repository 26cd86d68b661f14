"""nn.MultiheadAttention of gguf_train over the engine's attention.

Interface (kept so that the module is a drop-in): the constructor's arguments and the parameter
names and shapes (in_proj_weight or q/k/v_proj_weight, in_proj_bias, out_proj), Xavier-uniform
initialisation in that order, the forward's arguments and return value, the (L, E) / (L, B, E) /
(B, L, E) layouts, the mask conventions (True in a bool attn_mask or key_padding_mask = NOT attended,
turned into -1e9; float masks added) and the error messages of the reference
(gguf_train/nn/modules/transformer.py:21-191).

How it runs here:
* the in/out projections run on the repo's tcgen05 GEMM for bf16/f16 (functional.linear; fp32 on
  cuBLAS); self-attention with packed weights projects q, k and v with ONE GEMM over
  in_proj_weight and takes the heads as strided views of its output (no copies); the attention
  kernels read those views directly;
* attn_mask and key_padding_mask are merged into one additive mask, which the tensor-core kernels
  apply per 128 x 128 block (a key-padding mask costs almost nothing: only the blocks holding padded
  keys are read entry by entry);
* need_weights=False: scaled_dot_product_attention (the sm_100a path, forward and backward);
  need_weights=True: the output comes from the same fused kernels (which also return each row's
  log-sum-exp) and the returned weights from a kernel that turns the lse back into probabilities,
  with the same dropout decisions (functional.attention_weights); the reference instead forms the
  (B, heads, L, S) scores with matmul + softmax.
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
        E, heads = int(embed_dim), int(num_heads)
        self.embed_dim, self.num_heads = E, heads
        self.head_dim = E // heads
        assert self.head_dim * heads == E, "embed_dim must be divisible by num_heads"
        self.dropout = float(dropout)
        self.batch_first = bool(batch_first)
        self.kdim = E if kdim is None else int(kdim)
        self.vdim = E if vdim is None else int(vdim)
        self._qkv_same = self.kdim == E and self.vdim == E
        make = dict(device=device, dtype=dtype or torch.get_default_dtype())
        shapes = ({"in_proj_weight": (3 * E, E)} if self._qkv_same else
                  {"q_proj_weight": (E, E), "k_proj_weight": (E, self.kdim), "v_proj_weight": (E, self.vdim)})
        # registration (and so initialisation) order: in_proj_weight, q, k, v
        for name in ("in_proj_weight", "q_proj_weight", "k_proj_weight", "v_proj_weight"):
            if name in shapes:
                self.register_parameter(name, nn.Parameter(nn.init.xavier_uniform_(torch.empty(shapes[name], **make))))
            else:
                self.register_parameter(name, None)
        self.register_parameter("in_proj_bias", nn.Parameter(torch.zeros(3 * E, **make)) if bias else None)
        self.out_proj = nn.Linear(E, E, bias=bias, **make)

    # ---------------------------------------------------------------- forward

    def forward(self, query, key, value, key_padding_mask=None, need_weights: bool = True, attn_mask=None,
                average_attn_weights: bool = True, is_causal: bool = False):
        self_attention = query is key and key is value
        xq, xk, xv, kpm, unbatched = self._batch_major(query, key, value, key_padding_mask)
        B, L, S = xq.shape[0], xq.shape[1], xk.shape[1]
        bias = self._score_bias(attn_mask, kpm, B, L, S, xq.dtype)  # argument errors before any device work
        q, k, v = self._heads(xq, xk, xv, self_attention)
        scale = self.head_dim ** -0.5
        p_drop = self.dropout if self.training else 0.0
        if need_weights:
            # the output through the fused kernels, then the weights from the same lse and the same
            # dropout decisions by the weights kernel (no (B, heads, L, S) scores are formed)
            seed = F.dropout_seed() if p_drop else 0
            ctx, lse = F.FlashAttentionLseFn.apply(q, k, v, bias, scale, is_causal, p_drop, seed)
            weights = F.AttentionWeightsFn.apply(q, k, lse, bias, scale, is_causal, average_attn_weights, p_drop, seed)
        else:
            ctx = F.scaled_dot_product_attention(q, k, v, attn_mask=bias, dropout_p=p_drop, is_causal=is_causal,
                                                 scale=scale)
            weights = None
        y = F.linear(ctx.transpose(1, 2).reshape(B, L, self.embed_dim), self.out_proj.weight, self.out_proj.bias)
        if not self.batch_first:
            y = y.transpose(0, 1)
        if unbatched:
            y = y.squeeze(0 if self.batch_first else 1)
            weights = None if weights is None else weights.squeeze(0)
        return y, weights

    def _batch_major(self, query, key, value, key_padding_mask):
        """(B, L, E) views of the inputs whatever their layout, the key-padding mask as (B, S), and
        whether the call was unbatched."""
        ranks = (query.ndim, key.ndim, value.ndim)
        unbatched = query.ndim == 2
        if ranks not in ((3, 3, 3), (2, 2, 2)):
            raise RuntimeError(
                "MultiheadAttention: query, key and value must all be 3-D (batched) or all 2-D (unbatched), "
                f"got {query.ndim}-D, {key.ndim}-D and {value.ndim}-D"
            )
        if unbatched:
            if key_padding_mask is not None:
                if key_padding_mask.ndim != 1:
                    raise RuntimeError(
                        "MultiheadAttention: key_padding_mask of an unbatched input must be 1-D (S), "
                        f"got {list(key_padding_mask.shape)}"
                    )
                key_padding_mask = key_padding_mask[None]
            xs = [t[None] for t in (query, key, value)]
        elif self.batch_first:
            xs = [query, key, value]
        else:
            xs = [t.transpose(0, 1) for t in (query, key, value)]
        return xs[0], xs[1], xs[2], key_padding_mask, unbatched

    def _heads(self, xq, xk, xv, self_attention: bool):
        """Per-head q, k, v of shape (B, heads, len, head_dim). Self-attention with packed weights
        takes one GEMM over in_proj_weight; the heads are views of its (B, L, 3, heads, head_dim) output."""
        B, heads, hd = xq.shape[0], self.num_heads, self.head_dim
        if self_attention and self._qkv_same:
            qkv = F.linear(xq, self.in_proj_weight, self.in_proj_bias)
            q, k, v = qkv.reshape(B, xq.shape[1], 3, heads, hd).permute(2, 0, 3, 1, 4).unbind(0)
            return q, k, v
        if self._qkv_same:
            weights = self.in_proj_weight.chunk(3)
        else:
            weights = (self.q_proj_weight, self.k_proj_weight, self.v_proj_weight)
        biases = (None,) * 3 if self.in_proj_bias is None else self.in_proj_bias.chunk(3)
        return tuple(F.linear(x, w, bb).reshape(B, x.shape[1], heads, hd).transpose(1, 2)
                     for x, w, bb in zip((xq, xk, xv), weights, biases))

    def _score_bias(self, attn_mask, kpm, B: int, L: int, S: int, dtype):
        """attn_mask ((L, S) or (B*heads, L, S)) and key_padding_mask ((B, S)) as one additive mask
        that broadcasts against the scores (B, heads, L, S), or None."""
        bias = None
        if attn_mask is not None:
            if attn_mask.ndim == 2:
                if tuple(attn_mask.shape) != (L, S):
                    raise RuntimeError(
                        f"MultiheadAttention: the 2D attn_mask has shape {list(attn_mask.shape)}, expected {[L, S]}")
                bias = _additive(attn_mask, dtype, "attn_mask").reshape(1, 1, L, S)
            elif attn_mask.ndim == 3:
                want = [B * self.num_heads, L, S]
                if list(attn_mask.shape) != want:
                    raise RuntimeError(
                        f"MultiheadAttention: the 3D attn_mask has shape {list(attn_mask.shape)}, expected {want}")
                bias = _additive(attn_mask, dtype, "attn_mask").reshape(B, self.num_heads, L, S)
            else:
                raise RuntimeError(f"MultiheadAttention: attn_mask must be 2D or 3D, got {attn_mask.ndim}D")
        if kpm is not None:
            if tuple(kpm.shape) != (B, S):
                raise RuntimeError(
                    f"MultiheadAttention: key_padding_mask has shape {list(kpm.shape)}, expected {[B, S]}")
            pad = _additive(kpm, dtype, "key_padding_mask").reshape(B, 1, 1, S)
            bias = pad if bias is None else bias + pad
        return bias

    @staticmethod
    def _additive_mask(mask, dtype, name: str):
        """The reference's helper under its name (transformer.py:179-191): a mask as an additive one."""
        return _additive(mask, dtype, name)


def _additive(mask: torch.Tensor, dtype, name: str) -> torch.Tensor:
    """torch.nn convention: True in a bool mask = the position must NOT be attended, which becomes
    -1e9 (as the reference writes it); a float mask is added as it is, in the scores' dtype."""
    if mask.dtype == torch.bool:
        return torch.where(mask, -1e9, 0.0).to(dtype)
    if not mask.is_floating_point():
        raise RuntimeError(f"MultiheadAttention: {name} must be a boolean or floating point tensor, got {mask.dtype}")
    return mask.to(dtype)
