"""The reference-shaped handle ABI (include/gguf_train_attn.h) driven through ctypes exactly as the
reference's gguf_train/_C.py binds gt_flash_attention (:471-472), on CUDA tensors."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, seeded

pytestmark = pytest.mark.gpu


def _h(x, dtype):
    from gguf_train_b200 import _C
    from gguf_train_b200.handles import Handle

    if dtype == "bf16":
        return Handle.from_numpy(O.to_bits(x, O.BF16), _C.GT_BF16)
    return Handle.from_numpy(x.astype(np.float32))


def _back(h, dtype):
    a = h.to_numpy()
    return O.from_bits(a, O.BF16) if dtype == "bf16" else a.astype(np.float64)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_handle_forward_backward(dtype):
    from gguf_train_b200 import handles as H

    O.manual_seed(21)
    B, Hq, Hkv, L, D = 1, 4, 2, 150, 128
    s = 0.5 if dtype == "bf16" else 1.0
    q, k, v = seeded((B, Hq, L, D), dtype, s), seeded((B, Hkv, L, D), dtype, s), seeded((B, Hkv, L, D), dtype, s)
    g = seeded((B, Hq, L, D), dtype)
    hq, hk, hv, hg = _h(q, dtype), _h(k, dtype), _h(v, dtype), _h(g, dtype)
    tol = (2e-2, 1e-2) if dtype == "bf16" else (1e-4, 1e-4)
    out = H.flash_attention(hq, hk, hv, None, 0.0, True)
    assert_close(_back(out, dtype), O.sdpa_fwd(q, k, v, is_causal=True), *tol, "gt_flash_attention")
    out2, lse = H.flash_attention_fwd_lse(hq, hk, hv, None, 0.0, True)
    assert lse.shape == (B, Hq, L)
    dq, dk, dv = H.flash_attention_backward(hg, hq, hk, hv, None, out2, lse, 0.0, True)
    wq, wk, wv = O.sdpa_bwd(q, k, v, g, is_causal=True)
    for name, got, want in (("dq", dq, wq), ("dk", dk, wk), ("dv", dv, wv)):
        assert_close(_back(got, dtype), want, *(tol if dtype == "bf16" else (1e-3, 1e-3)), name)


def test_handle_errors_match_the_reference():
    from gguf_train_b200 import _C
    from gguf_train_b200 import handles as H

    q = H.Handle.from_numpy(np.zeros((2, 3, 4, 6), np.float32))
    k = H.Handle.from_numpy(np.zeros((2, 3, 5, 6), np.float32))
    for shape in ((2, 3), (5, 1, 1, 1), (4, 6)):
        m = H.Handle.from_numpy(np.ones(shape, np.bool_))
        with pytest.raises(RuntimeError, match="cannot be broadcast"):
            H.flash_attention(q, k, k, m)
    k2 = H.Handle.from_numpy(np.zeros((2, 2, 5, 6), np.float32))
    with pytest.raises(RuntimeError, match="num_heads must be divisible by num_kv_heads"):
        H.flash_attention(q, k2, k2)
    qc = H.Handle.from_numpy(np.zeros((2, 3, 4, 6), np.float32), device=_C.GT_DEV_CPU)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        H.flash_attention(qc, qc, qc)


def test_handle_quantize_and_decode():
    from gguf_train_b200 import _C
    from gguf_train_b200 import handles as H

    O.manual_seed(22)
    B, Hq, Hkv, S, D = 2, 8, 2, 600, 128
    kf = O.randn(B, Hkv, S, D).astype(np.float32)
    vf = O.randn(B, Hkv, S, D).astype(np.float32)
    hk = H.quantize(H.Handle.from_numpy(kf))
    hv = H.quantize(H.Handle.from_numpy(vf))
    assert hk.dtype == _C.GT_Q8_0 and hk.shape == (B, Hkv, S, D)
    assert np.array_equal(hk.to_numpy(), O.q8_0_quantize(kf))
    back = H.dequantize(hk, _C.GT_F32).to_numpy()
    assert np.array_equal(back, O.q8_0_dequantize(O.q8_0_quantize(kf), kf.shape))
    q = seeded((B, Hq, 1, D), "f16")
    hq = H.Handle.from_numpy(q.astype(np.float16))
    lens = np.array([600, 257], np.int32)
    out = H.flash_decode_q8_0(hq, hk, hv, H.Handle.from_numpy(lens))
    want = O.decode_q8_0(q, O.q8_0_quantize(kf), O.q8_0_quantize(vf), lens, Hkv, S)
    assert_close(out.to_numpy().astype(np.float64), want, 2e-2, 1e-2, "gt_flash_decode_q8_0")


def test_handle_rope_matches_oracle():
    """gt_rope and gt_rope_backward through handles, as the reference's RoPEFn calls them
    (_functions.py:1906-1919), with float positions converted to int32 as the reference does."""
    from gguf_train_b200 import _C
    from gguf_train_b200.handles import Handle
    import gguf_train_b200.handles as H

    O.manual_seed(91)
    x = seeded((2, 4, 24, 64), "f32")
    pos = ((np.arange(24) * 131 + 7) % 3000).astype(np.float32)
    hx, hp = _h(x, "f32"), Handle.from_numpy(pos)
    got = H.rope(hx, hp, 64, 2, 0, 10000.0, 1.0).to_numpy()
    back = H.rope(hx, hp, 64, 2, 0, 10000.0, 1.0, backward=True).to_numpy()
    assert _C.device_status() == 0
    assert_close(got, O.rope(x, pos.astype(np.int64), 64, 2), 2e-5, 1e-5, "gt_rope")
    assert_close(back, O.rope(x, pos.astype(np.int64), 64, 2, backward=True), 2e-5, 1e-5, "gt_rope_backward")


def test_reference_shaped_function_over_handles():
    """FlashAttentionFn as the reference's autograd engine runs it (gguf_train/_functions.py:1922-1965:
    forward(ctx, q, k, v, mask, scale, is_causal), backward(ctx, grad_out) -> six gradients), rewired to
    the engine as INTEGRATION.md shows: the forward saves the output and the log-sum-exp, the backward
    is one native call. Everything crosses the handle ABI (gt_tensor *), no torch tensor is involved;
    a bool (B, 1, L, S) key-padding mask, GQA and a causal mask, bf16."""
    import math

    from gguf_train_b200 import _C
    from gguf_train_b200 import handles as H

    class Context:  # what of the reference's Context the Function uses
        def save_for_backward(self, *tensors):
            self.saved_tensors = tensors

    class FlashAttentionFn:
        @staticmethod
        def forward(ctx, q, k, v, mask, scale, is_causal):
            ctx.scale = float(scale) if scale is not None else 1.0 / math.sqrt(q.shape[-1])
            ctx.is_causal = bool(is_causal)
            out, lse = H.flash_attention_fwd_lse(q, k, v, mask, ctx.scale, ctx.is_causal)
            ctx.save_for_backward(q, k, v, mask, out, lse)
            return out

        @staticmethod
        def backward(ctx, grad_out):
            q, k, v, mask, out, lse = ctx.saved_tensors
            dq, dk, dv = H.flash_attention_backward(grad_out, q, k, v, mask, out, lse, ctx.scale, ctx.is_causal)
            return dq, dk, dv, None, None, None

    O.manual_seed(23)
    B, Hq, Hkv, L, D = 2, 4, 2, 200, 128
    q, k, v = (seeded(s, "bf16", 0.5) for s in ((B, Hq, L, D), (B, Hkv, L, D), (B, Hkv, L, D)))
    g = seeded((B, Hq, L, D), "bf16")
    keep = np.ones((B, 1, 1, L), dtype=bool)
    keep[0, ..., 170:] = False  # the last 30 keys of sequence 0 are padding
    mh = H.Handle.from_numpy(keep.astype(np.uint8), _C.GT_BOOL)
    ctx = Context()
    out = FlashAttentionFn.forward(ctx, _h(q, "bf16"), _h(k, "bf16"), _h(v, "bf16"), mh, None, True)
    grads = FlashAttentionFn.backward(ctx, _h(g, "bf16"))
    assert grads[3:] == (None, None, None)
    m = np.broadcast_to(keep, (B, 1, L, L)).astype(np.float64)
    assert_close(_back(out, "bf16"), O.sdpa_fwd(q, k, v, m, True, is_causal=True), 2e-2, 1e-2, "forward")
    want = O.sdpa_bwd(q, k, v, g, m, True, is_causal=True)
    for name, got, w in zip(("dq", "dk", "dv"), grads[:3], want):
        assert_close(_back(got, "bf16"), w, 2e-2, 1e-2, name)
    assert _C.device_status() == 0
