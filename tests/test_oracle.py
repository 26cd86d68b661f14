"""The CPU oracle pinned against the golden fixtures, known answers and the reference tests' own
self-consistency checks (no GPU).

The reference cannot be built here (its ggml dependency is downloaded at build time), so the
oracle is pinned against independent implementations: gguf-py's Q8_0 codec (bit-exact with
ggml-quants.c by its own statement), torch's float64 SDPA and autograd, the C++ standard's
known answer for mt19937_64, and IEEE rounding as numpy/torch implement it.
"""

from __future__ import annotations

import math
import os

import numpy as np
import pytest

from oracle import mha as M
from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_mt19937_64_known_answer():
    # [rand.predef]: the 10000th output of a default-constructed mt19937_64 is 9981545732273789042
    assert int(O.engine_raw(5489, 10000)[-1]) == 9981545732273789042


def test_seeded_normals_are_reproducible_and_standard():
    O.manual_seed(0)
    a = O.randn(4096)
    O.manual_seed(0)
    assert np.array_equal(a, O.randn(4096))
    assert abs(a.mean()) < 0.05 and abs(a.std() - 1.0) < 0.05


def test_each_fill_uses_a_fresh_distribution():
    """gt_fill_normal builds a new normal_distribution per call (gt_core.cpp:1204): the polar method
    draws pairs, so a call of odd length drops its spare value and the next call starts on a new pair."""
    O.manual_seed(7)
    whole = O.randn(8)
    O.manual_seed(7)
    first, second = O.randn(3), O.randn(3)
    assert np.array_equal(first, whole[:3])
    assert np.array_equal(second, whole[4:7])


def test_dtype_rounding_matches_numpy_and_torch():
    import torch

    O.manual_seed(1)
    for scale in (1e-6, 1.0, 1e3, 7e4):
        y = O.randn(50000) * scale
        assert np.array_equal(O.to_bits(y, O.F16), y.astype(np.float32).astype(np.float16).view(np.uint16))
        want = torch.tensor(y, dtype=torch.float32).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
        assert np.array_equal(O.to_bits(y, O.BF16), want)
        assert np.array_equal(O.from_bits(O.to_bits(y, O.BF16), O.BF16), O.round_to(y, O.BF16))


def test_q8_0_matches_gguf_py_fixture():
    z = np.load(os.path.join(GOLDEN, "q8_0_gguf_py.npz"))
    assert np.array_equal(O.q8_0_quantize(z["x"]), z["blocks"])
    back = O.q8_0_dequantize(z["blocks"], z["x"].shape)
    rows = z["blocks"].reshape(-1, 34)
    d = rows[:, :2].copy().view(np.float16).astype(np.float32)
    qs = rows[:, 2:].view(np.int8).astype(np.float32)
    assert np.array_equal(back.reshape(-1, 32), qs * d)


def test_q8_0_matches_live_gguf_py():
    gguf = pytest.importorskip("gguf")
    from gguf.quants import quantize

    O.manual_seed(2)
    x = (O.randn(64, 256) * 2.5).astype(np.float32)
    assert np.array_equal(O.q8_0_quantize(x), quantize(x, gguf.GGMLQuantizationType.Q8_0).reshape(-1))


@pytest.mark.parametrize("name", ["gqa_causal", "lt_s_noncausal", "gt_s_causal", "bool_mask", "float_mask"])
def test_sdpa_matches_torch_fixture(name):
    z = np.load(os.path.join(GOLDEN, "sdpa_torch_f64.npz"))
    q, k, v, g = (z[f"{name}.{x}"] for x in "qkvg")
    causal = "causal" in name and "noncausal" not in name
    mask = z[f"{name}.mask"] if f"{name}.mask" in z.files else None
    is_bool = mask is not None and mask.dtype == np.bool_
    m = mask.astype(np.float64) if mask is not None else None
    # the fixture's torch run used the double scale; the oracle's forward takes the C float the
    # reference passes (gguf_train/_C.py:471), hence the 1e-7 tolerance
    out = O.sdpa_fwd(q, k, v, m, is_bool, scale=0.0, is_causal=causal)
    assert np.abs(out - z[f"{name}.out"]).max() < 1e-7
    dq, dk, dv = O.sdpa_bwd(q, k, v, g, m, is_bool, scale=1.0 / math.sqrt(q.shape[-1]), is_causal=causal)
    for got, key in ((dq, "dq"), (dk, "dk"), (dv, "dv")):
        assert np.abs(got - z[f"{name}.{key}"]).max() < 1e-9, key


def _composite(q, k, v, mask):
    """The reference tests' composite: softmax(q k^T / sqrt(D) masked) v
    (tests/test_pooling_and_attention.py:354-356), in float64 numpy."""
    s = q @ np.swapaxes(k, -1, -2) / math.sqrt(q.shape[-1])
    if mask is not None:
        s = np.where(mask, s, -np.inf) if mask.dtype == np.bool_ else s + mask
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    return (p / p.sum(-1, keepdims=True)) @ v


def test_reference_self_consistency_cases():
    """tests/test_pooling_and_attention.py:358-373 on the oracle: bool masks (True = attend) in every
    right-aligned broadcast and their -1e9 additive twins equal the composite within 1e-5."""
    rng = np.random.default_rng(6)
    q, k, v = rng.standard_normal((2, 3, 4, 6)), rng.standard_normal((2, 3, 5, 6)), rng.standard_normal((2, 3, 5, 6))
    base = rng.random((2, 3, 4, 5)) < 0.6
    base[..., 0] = True
    for mask in (base, base[:, :1], base[:1], base[0], base[0, 0], base[0, 0, :1], base[..., :1, :]):
        m4 = mask.reshape((1,) * (4 - mask.ndim) + mask.shape)
        want = _composite(q, k, v, np.broadcast_to(m4, (2, 3, 4, 5)))
        got = O.sdpa_fwd(q, k, v, m4.astype(np.float64), True, scale=float(np.float32(1 / math.sqrt(6))))
        assert np.abs(got - want).max() < 1e-5
        add = np.where(m4, 0.0, -1e9)
        got2 = O.sdpa_fwd(q, k, v, add, False, scale=float(np.float32(1 / math.sqrt(6))))
        assert np.abs(got2 - want).max() < 1e-5


def test_fully_masked_row_is_zero_and_causal_is_top_left():
    rng = np.random.default_rng(3)
    q, k, v = rng.standard_normal((1, 1, 3, 4)), rng.standard_normal((1, 1, 5, 4)), rng.standard_normal((1, 1, 5, 4))
    mask = np.ones((3, 5))
    mask[1] = 0
    out = O.sdpa_fwd(q, k, v, mask, True)
    assert np.all(out[0, 0, 1] == 0)  # gt_ops_nn.cpp:2509: inv = 0 when nothing is allowed
    causal = O.sdpa_fwd(q, k, v, is_causal=True)
    assert np.allclose(causal[0, 0, 0], v[0, 0, 0])  # row 0 sees key 0 only (s > l masked)


def test_decode_oracle_equals_dequantised_sdpa():
    O.manual_seed(4)
    B, H, Hkv, S, D = 2, 4, 2, 70, 64
    q = O.randn(B, H, 1, D)
    kf = O.randn(B, Hkv, S, D).astype(np.float32)
    vf = O.randn(B, Hkv, S, D).astype(np.float32)
    kq, vq = O.q8_0_quantize(kf), O.q8_0_quantize(vf)
    lens = np.array([70, 33], np.int32)
    got = O.decode_q8_0(q, kq, vq, lens, Hkv, S)
    kd = O.q8_0_dequantize(kq, kf.shape).astype(np.float64)
    vd = O.q8_0_dequantize(vq, vf.shape).astype(np.float64)
    for b in range(B):
        want = O.sdpa_fwd(q[b:b + 1], kd[b:b + 1, :, :lens[b]], vd[b:b + 1, :, :lens[b]])
        assert np.abs(got[b:b + 1] - want).max() < 1e-12


def test_mha_oracle_matches_torch_float64():
    import torch

    rng = np.random.default_rng(12)
    B, L, E, H = 2, 6, 8, 2
    x = rng.standard_normal((B, L, E))
    m = torch.nn.MultiheadAttention(E, H, batch_first=True, dtype=torch.float64)
    with torch.no_grad():
        m.in_proj_bias.copy_(torch.tensor(rng.standard_normal(3 * E) * 0.1))
        m.out_proj.bias.copy_(torch.tensor(rng.standard_normal(E) * 0.1))
    kpm = np.zeros((B, L), dtype=bool)
    kpm[1, -2:] = True
    am = np.triu(np.ones((L, L), dtype=bool), 1)
    tx = torch.tensor(x, requires_grad=True)
    want, _ = m(tx, tx, tx, key_padding_mask=torch.tensor(kpm), attn_mask=torch.tensor(am), need_weights=False)
    w_in = m.in_proj_weight.detach().numpy()
    b_in = m.in_proj_bias.detach().numpy()
    w_out = m.out_proj.weight.detach().numpy()
    b_out = m.out_proj.bias.detach().numpy()
    got, cache = M.forward(x, x, x, w_in, b_in, w_out, b_out, H, am, kpm)
    assert np.abs(got - want.detach().numpy()).max() < 1e-6
    g = rng.standard_normal((B, L, E))
    want.backward(torch.tensor(g))
    dxq, dxk, dxv, dw_in, db_in, dw_out, db_out = M.backward(g, cache)
    assert np.abs((dxq + dxk + dxv) - tx.grad.numpy()).max() < 1e-6
    assert np.abs(dw_in - m.in_proj_weight.grad.numpy()).max() < 1e-6
    assert np.abs(db_in - m.in_proj_bias.grad.numpy()).max() < 1e-6
    assert np.abs(dw_out - m.out_proj.weight.grad.numpy()).max() < 1e-9


def test_rope_oracle_properties():
    """The RoPE restatement: position 0 is the identity, each pair keeps its length, the backward
    undoes the forward, NeoX mode is normal mode on the interleaved dims, and dims past n_dims are
    copied; theta_scale is powf's correctly rounded value (0.7498942 for base 10000, n_dims 64)."""
    rs = np.random.RandomState(7)
    x = rs.randn(2, 3, 6, 16).astype(np.float32)
    pos = [0, 1, 5, 100, 4096, 7]
    y = O.rope(x, pos, 16)
    assert np.array_equal(y[:, :, 0], x[:, :, 0])
    pair = lambda a: a[..., 0::2] ** 2 + a[..., 1::2] ** 2  # noqa: E731
    assert np.allclose(pair(y), pair(x), rtol=1e-5, atol=1e-6)
    assert np.allclose(O.rope(y, pos, 16, backward=True), x, atol=1e-5)
    perm = np.concatenate([np.arange(0, 16, 2), np.arange(1, 16, 2)])  # interleaved -> halves
    yn = O.rope(x[..., perm], pos, 16, mode=2)
    assert np.allclose(yn, y[..., perm], atol=1e-6)
    yp = O.rope(x, pos, 8)
    assert np.array_equal(yp[..., 8:], x[..., 8:])
    # pair 1 at position 1 turns by exactly theta_scale
    e = np.zeros((1, 2, 64), np.float32)
    e[0, 1, 2] = 1.0
    assert O.rope(e, [0, 1], 64)[0, 1, 3] == np.float32(np.sin(np.float64(np.float32(0.7498942))))


def test_rope_oracle_matches_transformers_rotations():
    """The RoPE restatement against independent implementations of the two layouts: transformers'
    Llama apply_rotary_pos_emb (rotate_half: pairs i, i + d/2, ggml's NeoX mode) and GPT-J's
    (rotate_every_two: pairs 2i, 2i+1, ggml's normal mode), fed float64 angles p * base^(-2i/d).
    Positions stay small because ggml accumulates each angle in float32 (theta *= theta_scale), which
    drifts from the exact power by ~1e-6 relative at the last pairs: 1e-4 covers that at p < 16."""
    import torch
    from transformers.models.gptj.modeling_gptj import apply_rotary_pos_emb as gptj_rotary
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb as llama_rotary

    rs = np.random.RandomState(11)
    B, H, S, D, base = 2, 3, 16, 64, 10000.0
    x = rs.randn(B, H, S, D).astype(np.float32)
    pos = np.arange(S)
    inv = base ** (-np.arange(0, D, 2, dtype=np.float64) / D)
    ang = torch.tensor(pos[:, None] * inv[None, :])                  # (S, D/2) float64
    xt = torch.tensor(x, dtype=torch.float64)
    emb = torch.cat([ang, ang], dim=-1)[None]                        # (1, S, D)
    neox, _ = llama_rotary(xt, xt, emb.cos(), emb.sin(), unsqueeze_dim=1)
    assert np.allclose(O.rope(x, pos, D, mode=2, freq_base=base), neox.numpy(), atol=1e-4, rtol=0)
    gptj = gptj_rotary(xt.transpose(1, 2), ang.sin()[None], ang.cos()[None]).transpose(1, 2)
    assert np.allclose(O.rope(x, pos, D, mode=0, freq_base=base), gptj.numpy(), atol=1e-4, rtol=0)
