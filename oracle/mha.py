"""nn.MultiheadAttention restated in float64 numpy -- TEST INFRASTRUCTURE ONLY.

Follows the reference's MultiheadAttention.forward for batch_first inputs and need_weights=False
(gguf_train/nn/modules/transformer.py:70-191): in-projection by the three row blocks of
in_proj_weight plus bias, heads split as (B, H, L, D), bool masks turned into -1e9 additive masks
(_additive_mask :179-191), attn_mask (L, S) -> (1, 1, L, S), key_padding_mask (B, S) -> (B, 1, 1, S),
the two summed, scaled_dot_product_attention with scale 1/sqrt(D) (the oracle's restatement of
gt_flash_attention), heads merged, out-projection. The backward is the chain rule through those
steps, with the attention part from the oracle's restatement of FlashAttentionFn.backward.
"""

from __future__ import annotations

import math

import numpy as np

from . import oracle as O


def additive(mask: np.ndarray) -> np.ndarray:
    if mask.dtype == np.bool_:
        return np.where(mask, -1e9, 0.0)
    return mask.astype(np.float64)


def merged_mask(B, H, L, S, attn_mask=None, key_padding_mask=None):
    mask = None
    if attn_mask is not None:
        a = additive(attn_mask)
        mask = a.reshape(1, 1, L, S) if a.ndim == 2 else a.reshape(B, H, L, S)
    if key_padding_mask is not None:
        km = additive(key_padding_mask).reshape(B, 1, 1, S)
        mask = km if mask is None else mask + km
    if mask is not None:
        mask = np.ascontiguousarray(np.broadcast_to(mask, (B if mask.shape[0] > 1 else 1, mask.shape[1], L, S)))
    return mask


def forward(xq, xk, xv, w_in, b_in, w_out, b_out, H, attn_mask=None, key_padding_mask=None, is_causal=False):
    xq, xk, xv = (np.asarray(x, np.float64) for x in (xq, xk, xv))
    B, L, E = xq.shape
    S = xk.shape[1]
    D = E // H
    wq, wk, wv = w_in[:E], w_in[E:2 * E], w_in[2 * E:]
    bq, bk, bv = b_in[:E], b_in[E:2 * E], b_in[2 * E:]
    q = (xq @ wq.T + bq).reshape(B, L, H, D).transpose(0, 2, 1, 3)
    k = (xk @ wk.T + bk).reshape(B, S, H, D).transpose(0, 2, 1, 3)
    v = (xv @ wv.T + bv).reshape(B, S, H, D).transpose(0, 2, 1, 3)
    mask = merged_mask(B, H, L, S, attn_mask, key_padding_mask)
    scale = 1.0 / math.sqrt(D)
    a = O.sdpa_fwd(q, k, v, mask, False, scale=scale, is_causal=is_causal)
    merged = a.transpose(0, 2, 1, 3).reshape(B, L, E)
    out = merged @ w_out.T + b_out
    cache = dict(xq=xq, xk=xk, xv=xv, q=q, k=k, v=v, merged=merged, mask=mask, scale=scale, H=H,
                 w_in=w_in, w_out=w_out, is_causal=is_causal)
    return out, cache


def backward(dout, c):
    """Gradients (dxq, dxk, dxv, dw_in, db_in, dw_out, db_out) of sum(out * dout)."""
    dout = np.asarray(dout, np.float64)
    B, L, E = dout.shape
    S = c["xk"].shape[1]
    H = c["H"]
    D = E // H
    dw_out = dout.reshape(-1, E).T @ c["merged"].reshape(-1, E)
    db_out = dout.sum(axis=(0, 1))
    dmerged = dout @ c["w_out"]
    da = dmerged.reshape(B, L, H, D).transpose(0, 2, 1, 3)
    dq, dk, dv = O.sdpa_bwd(c["q"], c["k"], c["v"], da, c["mask"], False, scale=c["scale"], is_causal=c["is_causal"])
    dqp = dq.transpose(0, 2, 1, 3).reshape(B, L, E)
    dkp = dk.transpose(0, 2, 1, 3).reshape(B, S, E)
    dvp = dv.transpose(0, 2, 1, 3).reshape(B, S, E)
    w_in = c["w_in"]
    wq, wk, wv = w_in[:E], w_in[E:2 * E], w_in[2 * E:]
    dxq, dxk, dxv = dqp @ wq, dkp @ wk, dvp @ wv
    dw_in = np.concatenate([dqp.reshape(-1, E).T @ c["xq"].reshape(-1, E),
                            dkp.reshape(-1, E).T @ c["xk"].reshape(-1, E),
                            dvp.reshape(-1, E).T @ c["xv"].reshape(-1, E)], axis=0)
    db_in = np.concatenate([dqp.sum(axis=(0, 1)), dkp.sum(axis=(0, 1)), dvp.sum(axis=(0, 1))])
    return dxq, dxk, dxv, dw_in, db_in, dw_out, db_out
