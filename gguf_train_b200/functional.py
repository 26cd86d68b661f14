"""Attention functions of the engine: the gguf_train surface over the sm_100a kernels.

`scaled_dot_product_attention` and `FlashAttentionFn` keep the names, arguments, defaults, mask
rules and error messages of the reference (gguf_train/nn/functional.py:724-767,
gguf_train/_functions.py:1922-1965). Tensors are torch CUDA tensors; torch provides storage,
streams and autograd bookkeeping, while the forward and backward run in this package's native
library through its C ABI. A CPU tensor is an error: the engine has no CPU path.

Differences from the reference, by design:
* FlashAttentionFn saves the output and the per-row log-sum-exp and runs a fused backward
  instead of recomputing the probabilities with separate matmul/softmax ops. For a row in which
  every key is masked, the forward gives 0 (as the reference) and the backward gives zero
  gradients; the reference's op-by-op backward would instead differentiate a softmax over
  -1e9 scores there.
* Dropout (dropout_p > 0) runs inside the kernels: each keep/drop decision is a counter-based hash of
  (seed, batch-head, query, key), so the backward recomputes the forward's mask without storing it;
  the reference draws its mask from its sequential generator, so the masks differ, the semantics
  (inverted dropout on the softmax probabilities) do not.
"""

from __future__ import annotations

import ctypes
import math

import torch

from . import _C

_DTYPE_CODE = {
    torch.float32: _C.GT_F32,
    torch.float16: _C.GT_F16,
    torch.bfloat16: _C.GT_BF16,
    torch.float64: _C.GT_F64,
    torch.bool: _C.GT_BOOL,
}


def _code(t: torch.Tensor) -> int:
    try:
        return _DTYPE_CODE[t.dtype]
    except KeyError:
        raise RuntimeError(f"flash_attention: unsupported dtype {t.dtype}") from None


def _t4(t: torch.Tensor, shape=None, stride=None) -> _C.Tensor4:
    r = _C.Tensor4()
    r.data = t.data_ptr() if t.numel() else 0
    shp = tuple(t.shape) if shape is None else tuple(shape)
    std = tuple(t.stride()) if stride is None else tuple(stride)
    for i in range(4):
        r.shape[i] = int(shp[i])
        r.stride[i] = int(std[i])
    r.dtype = _code(t)
    return r


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _require_cuda(name: str, *ts) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError(
                f"{name}: this engine runs CUDA tensors only (got a {t.device} tensor); move it with .cuda()"
            )


def _native_mask(mask: torch.Tensor, B: int, H: int, L: int, S: int) -> _C.Tensor4:
    """The native layer's mask rule (gt_ops_nn.cpp:2437-2454): a 2-D (L|1, S|1) or 4-D
    (B|1, H|1, L|1, S|1) mask; size-1 dimensions broadcast."""
    want = (B, H, L, S)
    fits = mask.ndim in (2, 4) and all(m == 1 or m == w for m, w in zip(mask.shape, want[4 - mask.ndim:]))
    if not fits:
        raise RuntimeError(
            f"flash_attention: attn_mask of shape {list(mask.shape)} cannot be broadcast to the attention weights "
            f"{list(want)}"
        )
    shape = (1,) * (4 - mask.ndim) + tuple(mask.shape)
    stride = (0,) * (4 - mask.ndim) + tuple(mask.stride())
    stride = tuple(0 if s == 1 else st for s, st in zip(shape, stride))
    return _t4(mask, shape, stride)


def _opts(flags: int = 0, dropout_p: float = 0.0, seed: int = 0) -> _C.SdpaOpts:
    o = _C.SdpaOpts()
    o.flags, o.dropout_p, o.dropout_seed = int(flags), float(dropout_p), int(seed) & (2**64 - 1)
    return o


def dropout_seed() -> int:
    """A dropout seed drawn from torch's default generator (so torch.manual_seed makes it repeat)."""
    return int(torch.randint(0, 2**62, (), dtype=torch.int64).item())


def sdpa_forward(q, k, v, mask=None, scale: float | None = None, is_causal: bool = False, need_lse: bool = True,
                 out: torch.Tensor | None = None, dropout_p: float = 0.0, seed: int = 0):
    """One call of the native forward: returns (out, lse). lse is (B, H, L), float64 for float64
    inputs and float32 otherwise, or None. `out`, if given, is a (B, H, L, Dv) tensor or view of q's
    dtype on q's device that receives the result (any strides; it is returned). With dropout_p > 0 the
    attention probabilities are dropped with that probability (kept ones scaled by 1/(1-p)) by the
    counter-based decisions of `seed`; the lse is that of the undropped probabilities."""
    _require_cuda("flash_attention", q, k, v, mask)
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise RuntimeError("flash_attention expects 4D q, k, v tensors (B, H, L, D)")
    B, H, L, D = q.shape
    S, Dv = k.shape[2], v.shape[3]
    sc = (1.0 / math.sqrt(D)) if scale is None else float(scale)
    if out is None:
        out = torch.empty((B, H, L, Dv), dtype=q.dtype, device=q.device)
    lse_dt = torch.float64 if q.dtype == torch.float64 else torch.float32
    lse = torch.empty((B, H, L), dtype=lse_dt, device=q.device) if need_lse else None
    mt = _native_mask(mask, B, H, L, S) if mask is not None else None
    tq, tk, tv, to = _t4(q), _t4(k), _t4(v), _t4(out)
    opts = _opts(0, dropout_p, seed)
    rc = _C.lib.gtb_sdpa_fwd_ex(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv),
                                ctypes.byref(mt) if mt is not None else None, sc, 1 if is_causal else 0,
                                ctypes.byref(to), lse.data_ptr() if lse is not None and lse.numel() else None,
                                ctypes.byref(opts), _stream(q.device))
    _C.check_rc(rc, "flash_attention")
    return out, lse


def sdpa_forward_rope(q, k, v, positions, n_dims: int | None = None, mode: int = 0, freq_base: float = 10000.0,
                      freq_scale: float = 1.0, mask=None, scale: float | None = None, is_causal: bool = False,
                      need_lse: bool = True, k_positions: torch.Tensor | None = None, q_in_kernel: bool = False):
    """Prefill attention with RoPE in one call (gtb_sdpa_fwd_rope): returns (out, lse, k_rot) with
    out = attention(rope(q), rope(k), v) and k_rot = rope(k), bit for bit what rope() on q and k followed
    by sdpa_forward gives. `positions` (int32, one per query) are q's positions and, unless k_positions
    is given, k's too. k is rotated once into k_rot, which a caller keeps as its K cache; q into a
    scratch copy, or with q_in_kernel=True (tcgen05 kernel, no mask) in shared memory inside the kernel
    (no copy of q, slower on B200)."""
    _require_cuda("flash_attention (rope)", q, k, v, mask, positions, k_positions)
    if q.ndim != 4 or k.ndim != 4 or v.ndim != 4:
        raise RuntimeError("flash_attention (rope) expects 4D q, k, v tensors (B, H, L, D)")
    B, H, L, D = q.shape
    S, Dv = k.shape[2], v.shape[3]
    kp = positions if k_positions is None else k_positions
    for name, pt in (("positions", positions), ("k_positions", kp)):
        if pt.dtype != torch.int32 or pt.ndim != 1:
            raise RuntimeError(f"flash_attention (rope): {name} must be a 1-D int32 tensor")
    positions, kp = positions.contiguous(), kp.contiguous()
    q, k = q.contiguous(), k.contiguous()
    nd = D if n_dims is None else int(n_dims)
    sc = (1.0 / math.sqrt(D)) if scale is None else float(scale)
    out = torch.empty((B, H, L, Dv), dtype=q.dtype, device=q.device)
    k_rot = torch.empty_like(k)
    lse_dt = torch.float64 if q.dtype == torch.float64 else torch.float32
    lse = torch.empty((B, H, L), dtype=lse_dt, device=q.device) if need_lse else None
    mt = _native_mask(mask, B, H, L, S) if mask is not None else None
    tq, tk, tv, to, tkr = _t4(q), _t4(k), _t4(v), _t4(out), _t4(k_rot)
    rc = _C.lib.gtb_sdpa_fwd_rope(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv),
                                  ctypes.byref(mt) if mt is not None else None, sc, 1 if is_causal else 0,
                                  positions.data_ptr() if positions.numel() else None, positions.numel(),
                                  kp.data_ptr() if kp.numel() else None, kp.numel(), nd, int(mode), float(freq_base),
                                  float(freq_scale), 1 if q_in_kernel else 0, ctypes.byref(tkr), ctypes.byref(to),
                                  lse.data_ptr() if lse is not None and lse.numel() else None, _stream(q.device))
    _C.check_rc(rc, "flash_attention (rope)")
    return out, lse, k_rot


def sdpa_backward(grad_out, q, k, v, mask, out, lse, scale: float, is_causal: bool,
                  deterministic: bool | None = None, grads=None, dropout_p: float = 0.0, seed: int = 0):
    """One call of the native backward: returns (dq, dk, dv). With `deterministic` (default: whether
    torch.use_deterministic_algorithms is on) dq comes from the separate dq kernel and has the same
    bits on every run; otherwise, for head size 128, dq is summed with f32 reductions in global
    memory inside the dK/dV kernel (faster; the last bit may vary from run to run). `grads`, if given,
    is a (dq, dk, dv) triple of tensors or views shaped like q, k, v that receive the result.
    dropout_p and seed: those of the forward that produced `out` (its dropout mask is recomputed)."""
    if deterministic is None:
        deterministic = torch.are_deterministic_algorithms_enabled()
    B, H, L, D = q.shape
    S = k.shape[2]
    if grads is None:
        dq = torch.empty_like(q, memory_format=torch.contiguous_format)
        dk = torch.empty_like(k, memory_format=torch.contiguous_format)
        dv = torch.empty_like(v, memory_format=torch.contiguous_format)
    else:
        dq, dk, dv = grads
    if grad_out.dtype != q.dtype:
        grad_out = grad_out.to(q.dtype)
    mt = _native_mask(mask, B, H, L, S) if mask is not None else None
    tg, tq, tk, tv, to = _t4(grad_out), _t4(q), _t4(k), _t4(v), _t4(out)
    tdq, tdk, tdv = _t4(dq), _t4(dk), _t4(dv)
    rc = _C.lib.gtb_sdpa_bwd_ex(ctypes.byref(tg), ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv),
                                ctypes.byref(mt) if mt is not None else None, ctypes.byref(to),
                                lse.data_ptr() if lse.numel() else None, float(scale), 1 if is_causal else 0,
                                ctypes.byref(tdq), ctypes.byref(tdk), ctypes.byref(tdv),
                                ctypes.byref(_opts(_C.GTB_BWD_DETERMINISTIC if deterministic else 0, dropout_p, seed)),
                                _stream(q.device))
    _C.check_rc(rc, "flash_attention_backward")
    return dq, dk, dv


class FlashAttentionFn(torch.autograd.Function):
    """The autograd Function behind scaled_dot_product_attention (reference _functions.py:1922).

    apply(q, k, v, mask, scale, is_causal[, dropout_p]): q (B,H,L,D), k (B,Hkv,S,D), v (B,Hkv,S,Dv), mask
    None, (L,S) or 4-D, bool (True = may attend) or float (added); scale None -> 1/sqrt(D). dropout_p > 0
    (an addition of this engine) drops attention probabilities inside the kernels with a seed drawn
    from torch's generator, kept for the backward.

    The forward keeps what the backward needs to skip recomputing the softmax normaliser: the output
    and the per-row log-sum-exp (the reference keeps only the inputs and rebuilds the probabilities
    with separate ops, _functions.py:1934-1965)."""

    @staticmethod
    def forward(ctx, q, k, v, mask, scale, is_causal, dropout_p=0.0):
        opts = (1.0 / math.sqrt(q.shape[-1]) if scale is None else float(scale), bool(is_causal))
        drop = (float(dropout_p), dropout_seed() if dropout_p else 0)
        out, lse = sdpa_forward(q, k, v, mask, *opts, need_lse=True, dropout_p=drop[0], seed=drop[1])
        ctx.opts, ctx.drop = opts, drop
        ctx.save_for_backward(q, k, v, mask, out, lse)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        if grad_out is None:
            return (None,) * 7
        q, k, v, mask, out, lse = ctx.saved_tensors
        dq, dk, dv = sdpa_backward(grad_out, q, k, v, mask, out, lse, *ctx.opts, dropout_p=ctx.drop[0], seed=ctx.drop[1])
        return dq, dk, dv, None, None, None, None


class FlashAttentionLseFn(torch.autograd.Function):
    """FlashAttentionFn that also returns the per-row log-sum-exp (not differentiable) and takes the
    dropout seed from the caller: apply(q, k, v, mask, scale, is_causal, dropout_p, seed) ->
    (out, lse). MultiheadAttention uses it when it returns its attention weights, which are formed
    from the same lse and the same dropout decisions."""

    @staticmethod
    def forward(ctx, q, k, v, mask, scale, is_causal, dropout_p, seed):
        opts = (1.0 / math.sqrt(q.shape[-1]) if scale is None else float(scale), bool(is_causal))
        out, lse = sdpa_forward(q, k, v, mask, *opts, need_lse=True, dropout_p=float(dropout_p), seed=int(seed))
        ctx.opts, ctx.drop = opts, (float(dropout_p), int(seed))
        ctx.save_for_backward(q, k, v, mask, out, lse)
        ctx.mark_non_differentiable(lse)
        return out, lse

    @staticmethod
    def backward(ctx, grad_out, _grad_lse):
        if grad_out is None:
            return (None,) * 8
        q, k, v, mask, out, lse = ctx.saved_tensors
        dq, dk, dv = sdpa_backward(grad_out, q, k, v, mask, out, lse, *ctx.opts, dropout_p=ctx.drop[0], seed=ctx.drop[1])
        return dq, dk, dv, None, None, None, None, None


def attention_weights(q, k, lse, mask=None, scale: float | None = None, is_causal: bool = False,
                      average: bool = True, dropout_p: float = 0.0, seed: int = 0) -> torch.Tensor:
    """The attention probabilities of a forward that has run (its lse, mask, scale, causality and
    dropout seed), on the device: (B, L, S) averaged over heads, or (B, H, L, S); q's dtype. The
    need_weights=True output of MultiheadAttention (reference transformer.py:153-166), without the
    (B, H, L, S) scores of the reference's matmul + softmax."""
    _require_cuda("attention_weights", q, k, lse, mask)
    B, H, L, D = q.shape
    S = k.shape[2]
    sc = (1.0 / math.sqrt(D)) if scale is None else float(scale)
    out = torch.empty((B, 1 if average else H, L, S), dtype=q.dtype, device=q.device)
    mt = _native_mask(mask, B, H, L, S) if mask is not None else None
    tq, tk, to = _t4(q), _t4(k), _t4(out)
    rc = _C.lib.gtb_attn_weights(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(mt) if mt is not None else None,
                                 lse.data_ptr() if lse.numel() else None, sc, 1 if is_causal else 0,
                                 1 if average else 0, ctypes.byref(_opts(0, dropout_p, seed)), ctypes.byref(to),
                                 _stream(q.device))
    _C.check_rc(rc, "attention_weights")
    return out[:, 0] if average else out


def _keep_mask_torch(seed: int, p: float, B: int, H: int, L: int, S: int, device) -> torch.Tensor:
    """The kernels' dropout decisions (csrc/dropout.cuh: lowbias32 chained over seed, batch-head, row,
    key) in torch integer ops, for the recomputing backward of attention_weights."""
    M = 0xFFFFFFFF

    def h32(x):
        x = x ^ (x >> 16)
        x = (x * 0x7FEB352D) & M
        x = x ^ (x >> 15)
        x = (x * 0x846CA68B) & M
        return x ^ (x >> 16)

    thr = min(int(float(torch.tensor(p, dtype=torch.float32)) * 4294967296.0), M)
    bh = torch.arange(B * H, device=device, dtype=torch.int64)
    head = h32(((seed >> 32) & M) ^ h32((seed & M) ^ bh))
    row = h32(head[:, None] ^ torch.arange(L, device=device, dtype=torch.int64)[None])
    x = h32((row[:, :, None] + torch.arange(S, device=device, dtype=torch.int64)[None, None]) & M)
    return (x >= thr).view(B, H, L, S)


class AttentionWeightsFn(torch.autograd.Function):
    """attention_weights as an autograd Function: apply(q, k, lse, mask, scale, is_causal, average,
    dropout_p, seed). The forward is the native kernel. Gradients reach q and k only when the caller
    differentiates through the returned weights (rare: they are usually inspected); the backward then
    recomputes the probabilities with torch ops (scores, softmax, the same dropout decisions) and
    differentiates those."""

    @staticmethod
    def forward(ctx, q, k, lse, mask, scale, is_causal, average, dropout_p, seed):
        ctx.args = (scale, bool(is_causal), bool(average), float(dropout_p), int(seed))
        ctx.save_for_backward(q, k, mask)
        return attention_weights(q, k, lse, mask, scale, is_causal, average, dropout_p, seed)

    @staticmethod
    def backward(ctx, grad_w):
        q, k, mask = ctx.saved_tensors
        scale, causal, average, p, seed = ctx.args
        with torch.enable_grad():
            qd, kd = q.detach().requires_grad_(), k.detach().requires_grad_()
            B, H, L, D = q.shape
            S, group = k.shape[2], H // k.shape[1]
            sc = (1.0 / math.sqrt(D)) if scale is None else float(scale)
            logits = torch.matmul(qd.float(), kd.float().repeat_interleave(group, dim=1).transpose(2, 3)) * sc
            if causal:
                logits = logits.masked_fill(torch.ones((L, S), dtype=torch.bool, device=q.device).triu(1), float("-inf"))
            if mask is not None:
                logits = logits.masked_fill(mask.logical_not(), float("-inf")) if mask.dtype == torch.bool \
                    else logits + mask.float()
            probs = torch.softmax(logits, dim=3)
            if p > 0.0:
                probs = probs * _keep_mask_torch(seed, p, B, H, L, S, q.device) / (1.0 - p)
            w = probs.mean(dim=1) if average else probs
            dq, dk = torch.autograd.grad(w, (qd, kd), grad_w.float())
        return dq.to(q.dtype), dk.to(k.dtype), None, None, None, None, None, None, None


def _autocast_lower(*ts):
    """Inside torch.autocast, floating arguments are cast to the autocast dtype, as the reference's
    _autocast_op(_AUTOCAST_LOWER) does for SDPA (gguf_train/_tensor.py:261-282)."""
    if not torch.is_autocast_enabled("cuda"):
        return ts, False
    dt = torch.get_autocast_dtype("cuda")
    return tuple(t.to(dt) if (t is not None and t.is_floating_point()) else t for t in ts), True


def _as_4d_mask(mask: torch.Tensor, query: torch.Tensor, key: torch.Tensor) -> torch.Tensor:
    """A mask of rank <= 4 lined up against the attention weights (B, H, L, S) from the right; each
    of its dimensions must be 1 or the full size (the reference's rule, nn/functional.py:735-746).
    Returns it as a 4-D view."""
    if query.ndim != 4 or key.ndim != 4:
        return mask  # the native call reports the shape error
    target = (query.shape[0], query.shape[1], query.shape[2], key.shape[2])
    lead = 4 - mask.ndim
    padded = (1,) * max(lead, 0) + tuple(mask.shape)
    if lead < 0 or any(size not in (1, full) for size, full in zip(padded, target)):
        raise RuntimeError(
            f"scaled_dot_product_attention: attn_mask of shape {list(mask.shape)} cannot be broadcast "
            f"to the attention weights {list(target)}"
        )
    return mask if lead == 0 else mask.reshape(padded)  # leading size-1 dimensions: a view


def scaled_dot_product_attention(
    query: torch.Tensor,
    key: torch.Tensor,
    value: torch.Tensor,
    attn_mask: torch.Tensor | None = None,
    dropout_p: float = 0.0,
    is_causal: bool = False,
    scale: float | None = None,
    enable_gqa: bool = False,
) -> torch.Tensor:
    """torch.nn.functional.scaled_dot_product_attention, as gguf_train defines it
    (nn/functional.py:724-767): a bool mask marks keys that MAY be attended, a float mask is added,
    masks broadcast from the right against (B, H, L, S), GQA applies whenever H % Hkv == 0
    (`enable_gqa` changes nothing), causal masking is top-left aligned. The call is FlashAttentionFn on
    the sm_100a kernels, dropout included (dropout_p > 0: the probabilities are dropped inside the
    kernels, with the reference's semantics; the mask is drawn from a counter-based hash seeded from
    torch's generator instead of the reference's sequential generator)."""
    del enable_gqa
    lowered, cast = _autocast_lower(query, key, value, attn_mask)
    if cast:
        with torch.autocast("cuda", enabled=False):
            return scaled_dot_product_attention(*lowered, dropout_p, is_causal, scale)
    sc = 1.0 / math.sqrt(query.shape[-1]) if scale is None else float(scale)
    mask = None if attn_mask is None else _as_4d_mask(attn_mask, query, key)
    if dropout_p != 0.0:
        return FlashAttentionFn.apply(query, key, value, mask, sc, is_causal, float(dropout_p))
    return FlashAttentionFn.apply(query, key, value, mask, sc, is_causal)


def sdpa_from_host(query: torch.Tensor, key: torch.Tensor, value: torch.Tensor, out: torch.Tensor | None = None,
                   attn_mask: torch.Tensor | None = None, is_causal: bool = False, scale: float | None = None,
                   chunk: int | None = None, device=None) -> torch.Tensor:
    """Scaled dot-product attention of q (B, H, L, D), k (B, Hkv, S, D), v (B, Hkv, S, Dv) held in host
    memory (pinned, for the copies to be asynchronous), computed on the GPU by the native
    gtb_sdpa_fwd_host; the result lands in `out` (host, (B, H, L, Dv), pinned and allocated when not
    given), which is returned.

    The work is cut into ceil(B / chunk) pieces when `chunk` is given, else 8 (whole sequences when
    the batch has that many, otherwise each sequence's kv heads in groups, with their query heads).
    Piece i's q, k, v are copied to the device on one internal stream while piece i-1 is attended on
    the caller's current stream and piece i-2's output is copied back on another, so both directions
    of PCIe are busy at once and the kernels run behind the copies. Like any non_blocking copy, `out`
    is complete once the caller's current stream has passed this call (e.g. after
    torch.cuda.current_stream().synchronize()). Masks are not taken here: copy the tensors and use
    scaled_dot_product_attention."""
    if attn_mask is not None:
        raise RuntimeError("sdpa_from_host: attn_mask is not supported; copy the tensors to the GPU and use "
                           "scaled_dot_product_attention")
    for name, t in (("query", query), ("key", key), ("value", value), ("out", out)):
        if t is not None and t.device.type != "cpu":
            raise RuntimeError(f"sdpa_from_host: {name} must be in host memory (got {t.device}); for CUDA tensors "
                               f"use scaled_dot_product_attention")
    if query.ndim != 4 or key.ndim != 4 or value.ndim != 4:
        raise RuntimeError("flash_attention expects 4D q, k, v tensors (B, H, L, D)")
    B, H, L, D = query.shape
    Dv = value.shape[3]
    if key.shape[0] != B or value.shape[0] != B:
        raise RuntimeError("sdpa_from_host: q, k, v must have the same batch size")
    if out is None:
        out = torch.empty((B, H, L, Dv), dtype=query.dtype, pin_memory=True)
    elif tuple(out.shape) != (B, H, L, Dv) or out.dtype != query.dtype or not out.is_contiguous():
        raise RuntimeError(f"sdpa_from_host: out must be a contiguous {(B, H, L, Dv)} tensor of {query.dtype}")
    if out.numel() == 0:
        return out
    q, k, v = (t.contiguous() for t in (query, key, value))
    pieces = -(-B // chunk) if chunk else 0
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        tq, tk, tv, to = _t4(q), _t4(k), _t4(v), _t4(out)
        rc = _C.lib.gtb_sdpa_fwd_host(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tv),
                                      -1.0 if scale is None else float(scale), 1 if is_causal else 0,
                                      ctypes.byref(to), pieces, torch.cuda.current_stream(dev).cuda_stream)
    _C.check_rc(rc, "flash_attention")
    return out


# ------------------------------------------------------------------ linear layers (MHA projections)

def _linear_2d(a: torch.Tensor, b: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    """c = a b^T (+ bias) on the tensor-core GEMM: a (M, K), b (N, K) contiguous 16-bit CUDA tensors."""
    M, K = a.shape
    N = b.shape[0]
    c = torch.empty((M, N), dtype=a.dtype, device=a.device)
    rc = _C.lib.gtb_linear(a.data_ptr(), b.data_ptr(), bias.data_ptr() if bias is not None else None, c.data_ptr(),
                           M, N, K, K, K, N, _code(a), _stream(a.device))
    _C.check_rc(rc, "linear")
    return c


class LinearFn(torch.autograd.Function):
    """F.linear(x, weight, bias) for bf16/f16 on the repo's tcgen05 GEMM (gtb_linear), the role of
    gt_linear (reference csrc/gt_ops_nn.cpp:256-335). Backward: dx = dy W and dW = dy^T x are the same
    kernel on transposed copies (both operands K-major), db = the column sums of dy."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        lead = x.shape[:-1]
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        w = weight.contiguous()
        y = _linear_2d(x2, w, bias.contiguous() if bias is not None else None)
        ctx.save_for_backward(x2, w)
        ctx.has_bias = bias is not None
        return y.view(*lead, w.shape[0])

    @staticmethod
    def backward(ctx, gy):
        x2, w = ctx.saved_tensors
        g2 = gy.reshape(-1, w.shape[0]).contiguous()
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            dx = _linear_2d(g2, w.t().contiguous(), None).view(*gy.shape[:-1], w.shape[1])
        if ctx.needs_input_grad[1]:
            dw = _linear_2d(g2.t().contiguous(), x2.t().contiguous(), None)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            db = g2.float().sum(0).to(g2.dtype)
        return dx, dw, db


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """F.linear on the engine: bf16/f16 on the tensor-core GEMM (LinearFn); other dtypes (fp32: there
    is no repo fp32 GEMM to beat cuBLAS's on the CUDA cores) and leading sizes that are not multiples
    of 8 through torch.nn.functional.linear."""
    _require_cuda("linear", x, weight, bias)
    K, N = x.shape[-1], weight.shape[0]
    if x.dtype in (torch.bfloat16, torch.float16) and weight.dtype == x.dtype and \
            (bias is None or bias.dtype == x.dtype) and K % 8 == 0 and N % 8 == 0 and K > 0 and x.numel() > 0:
        return LinearFn.apply(x, weight, bias)
    return torch.nn.functional.linear(x, weight, bias)


# ------------------------------------------------------------------ Q8_0 KV cache

def quantize_q8_0(x: torch.Tensor) -> torch.Tensor:
    """GGUF Q8_0 blocks of a CUDA tensor (rows along the last dim), as uint8 of shape
    (..., last/32*34). Bit-exact with ggml's reference quantiser (gt_quantize, reference
    csrc/gt_ops_extra.cpp:2002)."""
    _require_cuda("quantize", x)
    if x.shape[-1] % 32:
        raise RuntimeError("Tensor size must be a multiple of ggml quantization block size")
    x = x.contiguous()
    out = torch.empty(tuple(x.shape[:-1]) + (x.shape[-1] // 32 * 34,), dtype=torch.uint8, device=x.device)
    row = x.shape[-1]
    rc = _C.lib.gtb_q8_0_quantize(x.data_ptr() if x.numel() else None, _code(x), x.numel() // max(row, 1), row,
                                  out.data_ptr() if out.numel() else None, _stream(x.device))
    _C.check_rc(rc, "quantize")
    return out


def q8_0_append(cache: torch.Tensor, x: torch.Tensor, pos: torch.Tensor, advance: bool = True,
                rope: dict | None = None) -> torch.Tensor:
    """Append new rows to a Q8_0 KV cache on the device: x (B, Hkv, n_new, D) is quantised (bit for bit
    as quantize_q8_0) into rows pos[b] .. pos[b] + n_new - 1 of cache (B, Hkv, Smax, D/32*34) uint8,
    the layout decode_q8_0 reads; pos (B) int32 holds the sequences' current lengths (decode_q8_0's
    seq_lens) and, with `advance`, is increased by n_new afterwards. With `rope` (a dict of rope()'s
    n_dims, mode, freq_base, freq_scale) each row is first rotated for its cache position, in f32.
    Rows that would fall outside the cache are skipped and leave status 60 in the device status word
    (_C.device_status()). Returns cache."""
    _require_cuda("q8_0_append", cache, x, pos)
    if x.ndim != 4 or cache.ndim != 4:
        raise RuntimeError("q8_0_append: x must be (B, Hkv, n_new, D) and cache (B, Hkv, Smax, D/32*34)")
    B, Hkv, n_new, D = x.shape
    if D % 32:
        raise RuntimeError("Tensor size must be a multiple of ggml quantization block size")
    if cache.dtype != torch.uint8 or tuple(cache.shape[:2]) != (B, Hkv) or cache.shape[3] != D // 32 * 34 \
            or not cache.is_contiguous():
        raise RuntimeError(f"q8_0_append: cache must be a contiguous uint8 tensor ({B}, {Hkv}, Smax, {D // 32 * 34})")
    if pos.dtype != torch.int32 or tuple(pos.shape) != (B,) or not pos.is_contiguous():
        raise RuntimeError(f"q8_0_append: pos must be a contiguous int32 tensor of shape ({B},)")
    x = x.contiguous()
    args = (x.data_ptr() if x.numel() else None, _code(x), B, Hkv, n_new, D,
            cache.data_ptr() if cache.numel() else None, cache.shape[2],
            pos.data_ptr() if pos.numel() else None, 1 if advance else 0)
    if rope is None:
        rc = _C.lib.gtb_q8_0_append(*args, _stream(x.device))
    else:
        r = {"n_dims": D, "mode": 0, "freq_base": 10000.0, "freq_scale": 1.0}
        r.update(rope)
        rc = _C.lib.gtb_q8_0_append_rope(*args, int(r["n_dims"]), int(r["mode"]), float(r["freq_base"]),
                                         float(r["freq_scale"]), _stream(x.device))
    _C.check_rc(rc, "q8_0_append")
    return cache


def _rope_run(x, positions, n_dims, mode, freq_base, freq_scale, backward):
    _require_cuda("rope", x, positions)
    if x.ndim < 3 or x.ndim > 4:
        raise RuntimeError(f"rope: expected x of shape (batch, heads, seq_len, head_dim) or (heads, seq_len, head_dim), "
                           f"got {list(x.shape)}")
    if x.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise RuntimeError("rope: x must be f32, f16 or bf16")
    if positions.ndim != 1:
        raise RuntimeError(f"rope: pos must be a 1-D tensor with a position for each of the {x.shape[-2]} sequence "
                           f"elements, got shape {list(positions.shape)}")
    B = x.shape[0] if x.ndim == 4 else 1
    H, S, D = x.shape[-3], x.shape[-2], x.shape[-1]
    x = x.contiguous()
    pos = positions.to(torch.int32).contiguous()
    out = torch.empty_like(x)
    rc = _C.lib.gtb_rope(x.data_ptr() if x.numel() else None, _code(x), B, H, S, D,
                         pos.data_ptr() if pos.numel() else None, pos.numel(), int(n_dims), int(mode),
                         float(freq_base), float(freq_scale), 1 if backward else 0,
                         out.data_ptr() if out.numel() else None, _stream(x.device))
    _C.check_rc(rc, "rope")
    return out


class RoPEFn(torch.autograd.Function):
    """gguf_train's RoPEFn (_functions.py:1906-1919): forward gt_rope, backward gt_rope_backward (the
    rotation by -angle), both on the device."""

    @staticmethod
    def forward(ctx, x, pos, n_dims: int, mode: int, n_ctx_orig: int, freq_base: float, freq_scale: float):
        ctx.args = (n_dims, mode, float(freq_base), float(freq_scale))
        ctx.save_for_backward(pos)
        return _rope_run(x, pos, n_dims, mode, freq_base, freq_scale, False)

    @staticmethod
    def backward(ctx, grad_out):
        (pos,) = ctx.saved_tensors
        n_dims, mode, fb, fs = ctx.args
        return _rope_run(grad_out, pos, n_dims, mode, fb, fs, True), None, None, None, None, None, None


def rope(input: torch.Tensor, positions: torch.Tensor, n_dims: int | None = None, mode: int = 0, n_ctx_orig: int = 0,
         freq_base: float = 10000.0, freq_scale: float = 1.0) -> torch.Tensor:
    """gguf_train's F.rope (nn/functional.py:770-772) on CUDA tensors: rotary position embedding of x
    (B, H, S, D) or (H, S, D) with one position per sequence element (n_ctx_orig is accepted and, as
    with ggml's ext_factor 0 that the reference passes, has no effect)."""
    nd = input.shape[-1] if n_dims is None else int(n_dims)
    return RoPEFn.apply(input, positions, nd, int(mode), int(n_ctx_orig), float(freq_base), float(freq_scale))


def dequantize_q8_0(blocks: torch.Tensor, dtype=torch.float32) -> torch.Tensor:
    """Inverse of quantize_q8_0: x = q * d, in `dtype`."""
    _require_cuda("dequantize", blocks)
    if blocks.shape[-1] % 34:
        raise RuntimeError("dequantize: the last dimension must hold whole 34-byte Q8_0 blocks")
    row = blocks.shape[-1] // 34 * 32
    out = torch.empty(tuple(blocks.shape[:-1]) + (row,), dtype=dtype, device=blocks.device)
    blocks = blocks.contiguous()
    rc = _C.lib.gtb_q8_0_dequantize(blocks.data_ptr() if blocks.numel() else None, out.numel() // max(row, 1), row,
                                    out.data_ptr() if out.numel() else None, _DTYPE_CODE[dtype], _stream(out.device))
    _C.check_rc(rc, "dequantize")
    return out


def decode_q8_0(q: torch.Tensor, k_q8: torch.Tensor, v_q8: torch.Tensor, seq_lens: torch.Tensor,
                scale: float | None = None) -> torch.Tensor:
    """One decode step: q (B, H, 1, D) against Q8_0 caches k_q8, v_q8 of shape (B, Hkv, Smax, D/32*34)
    (uint8, from quantize_q8_0), sequence b attending its first seq_lens[b] rows. Returns (B, H, 1, D)
    in q's dtype. Equivalent to dequantising the caches and calling scaled_dot_product_attention."""
    _require_cuda("flash_decode_q8_0", q, k_q8, v_q8, seq_lens)
    B, H, Lq, D = q.shape
    if Lq != 1:
        raise RuntimeError("flash_decode_q8_0: q must be (B, H, 1, D)")
    if k_q8.ndim != 4 or k_q8.shape != v_q8.shape or k_q8.shape[0] != B or k_q8.shape[3] != D // 32 * 34:
        raise RuntimeError("flash_decode_q8_0: k and v caches must be (B, Hkv, Smax, D/32*34) uint8 Q8_0 rows")
    if seq_lens.dtype != torch.int32 or seq_lens.shape != (B,):
        raise RuntimeError("flash_decode_q8_0: seq_lens must be an int32 (B) tensor")
    Hkv, Smax = k_q8.shape[1], k_q8.shape[2]
    q = q.contiguous()
    k_q8 = k_q8.contiguous()
    v_q8 = v_q8.contiguous()
    seq_lens = seq_lens.contiguous()
    out = torch.empty_like(q)
    sc = 0.0 if scale is None else float(scale)
    rc = _C.lib.gtb_decode_q8_0(q.data_ptr(), _code(q), k_q8.data_ptr() if k_q8.numel() else None,
                                v_q8.data_ptr() if v_q8.numel() else None, seq_lens.data_ptr(), B, H, Hkv, Smax, D,
                                sc, out.data_ptr(), _stream(q.device))
    _C.check_rc(rc, "flash_decode_q8_0")
    return out
