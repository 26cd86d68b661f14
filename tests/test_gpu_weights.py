"""MultiheadAttention's need_weights=True output on the engine: the attention weights formed by the
weights kernel from the fused forward's lse (functional.attention_weights), against the reference's
explicit softmax (gguf_train/nn/modules/transformer.py:153-166) restated in float64: head-averaged
and per-head, causal, masks, GQA, dropout with the kernels' decisions, and gradients through the
returned weights."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, seeded, to_dev

pytestmark = pytest.mark.gpu


def _probs(q, k, mask, is_bool, scale, causal):
    B, H, L, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    ke = np.repeat(k, H // Hkv, axis=1)
    s = np.einsum("bhld,bhsd->bhls", q, ke) * scale
    if causal:
        s = s + np.where(np.arange(S)[None, :] > np.arange(L)[:, None], -np.inf, 0.0)
    if mask is not None:
        m = np.broadcast_to(mask, (B, H, L, S))
        s = np.where(m == 0, -np.inf, s) if is_bool else s + m
    s = s - s.max(-1, keepdims=True)
    p = np.exp(s)
    return p / p.sum(-1, keepdims=True)


@pytest.mark.parametrize("dt,B,H,Hkv,L,S,D,causal,kind,average", [
    ("bf16", 2, 4, 2, 200, 200, 128, True, None, True),
    ("bf16", 1, 4, 4, 130, 190, 64, False, "kpm", False),
    ("f32", 2, 8, 8, 64, 64, 64, False, "float", True),
    ("f32", 2, 4, 2, 100, 130, 64, True, None, False),   # fp32 tiled kernel: causal, GQA, every head, S % 4 != 0
    ("f32", 1, 4, 1, 97, 200, 64, False, "kpm", True),   # fp32 tiled kernel: bool mask read 4 keys per load
    ("f16", 1, 2, 1, 40, 70, 32, True, None, False),
    ("bf16", 2, 4, 1, 300, 256, 128, False, "float", True),  # tcgen05 kernel: float mask, 16-byte stores
    ("f16", 1, 4, 2, 260, 264, 64, True, None, False),       # tcgen05 kernel: causal, every head
    ("f64", 1, 2, 2, 17, 23, 8, False, "float", True),
])
def test_weights_match_the_explicit_softmax(dt, B, H, Hkv, L, S, D, causal, kind, average):
    import torch

    from gguf_train_b200 import functional as Fn

    O.manual_seed(B * 100 + L)
    q, k, v = seeded((B, H, L, D), dt, 0.5), seeded((B, Hkv, S, D), dt, 0.5), seeded((B, Hkv, S, D), dt, 0.5)
    mask = mt = None
    is_bool = kind == "kpm"
    if kind == "kpm":
        mask = np.ones((B, 1, 1, S))
        mask[..., S - 17:] = 0
        mt = torch.tensor(mask != 0).cuda()
    elif kind == "float":
        mask = O.round_to(O.randn(1, 1, L, S), {"bf16": O.BF16, "f16": O.F16, "f32": O.F32, "f64": O.F64}[dt])
        mask[0, 0, O.rand(L, S) < 0.1] = -np.inf
        mask[..., 0] = 0.0
        mt = to_dev(mask, dt)
    scale = D ** -0.5
    tq, tk, tv = (to_dev(x, dt) for x in (q, k, v))
    out, lse = Fn.sdpa_forward(tq, tk, tv, mt, scale, causal)
    w = Fn.attention_weights(tq, tk, lse, mt, scale, causal, average)
    P = _probs(q, k, mask, is_bool, float(np.float32(scale)), causal)
    want = P.mean(1) if average else P
    tol = {"bf16": (1e-2, 2e-2), "f16": (2e-3, 1e-2), "f32": (1e-5, 1e-4), "f64": (1e-7, 1e-7)}[dt]
    assert_close(w, want, *tol, f"weights {dt} average={average}")


def test_mha_need_weights_matches_the_reference_module():
    """nn.MultiheadAttention(need_weights=True), the default call, on the engine: output, averaged
    weights and input gradients against the float64 restatement, with attn_mask + key_padding_mask;
    and gradients that flow through the returned weights."""
    import torch

    import gguf_train_b200 as gtb
    from oracle import mha as M

    E, H, L, B = 64, 4, 48, 3
    torch.manual_seed(1)
    m = gtb.MultiheadAttention(E, H, batch_first=True, device="cuda", dtype=torch.float64)
    O.manual_seed(2)
    x = O.randn(B, L, E)
    am = np.where(O.bernoulli(L, L, p=0.1) > 0, -np.inf, 0.0)
    am[:, 0] = 0.0
    kpm = np.zeros((B, L), dtype=bool)
    kpm[1, L - 5:] = True
    tx = torch.tensor(x, device="cuda", requires_grad=True)
    out, w = m(tx, tx, tx, key_padding_mask=torch.tensor(kpm).cuda(), attn_mask=torch.tensor(am).cuda())
    assert w.shape == (B, L, L)
    w_in = m.in_proj_weight.detach().cpu().numpy()
    b_in = m.in_proj_bias.detach().cpu().numpy()
    want_out, _ = M.forward(x, x, x, w_in, b_in, m.out_proj.weight.detach().cpu().numpy(),
                            m.out_proj.bias.detach().cpu().numpy(), H, am, kpm)
    assert_close(out, want_out, 1e-7, 1e-7, "need_weights output")
    # weights: the softmax of the reference's scores, averaged over heads
    Wq, Wk = np.split(w_in, 3)[:2]
    bq, bk = np.split(b_in, 3)[:2]
    qh = (x @ Wq.T + bq).reshape(B, L, H, E // H).transpose(0, 2, 1, 3)
    kh = (x @ Wk.T + bk).reshape(B, L, H, E // H).transpose(0, 2, 1, 3)
    bias = am[None, None] + np.where(kpm, -1e9, 0.0)[:, None, None, :]
    want_w = _probs(qh, kh, bias, False, (E // H) ** -0.5, False).mean(1)
    assert_close(w, want_w, 1e-9, 1e-7, "need_weights weights")
    # gradients through the returned weights reach the input: a finite-difference check of them
    assert torch.autograd.gradcheck(lambda a: m(a, a, a)[1],
                                    (torch.tensor(x[:1, :6], device="cuda", requires_grad=True),),
                                    eps=1e-6, atol=1e-6, rtol=1e-4)
    # and the output's gradient with need_weights=True equals the need_weights=False one
    tx1 = torch.tensor(x, device="cuda", requires_grad=True)
    m(tx1, tx1, tx1, key_padding_mask=torch.tensor(kpm).cuda(), attn_mask=torch.tensor(am).cuda())[0].sum().backward()
    tx2 = torch.tensor(x, device="cuda", requires_grad=True)
    m(tx2, tx2, tx2, key_padding_mask=torch.tensor(kpm).cuda(), attn_mask=torch.tensor(am).cuda(),
      need_weights=False)[0].sum().backward()
    torch.testing.assert_close(tx1.grad, tx2.grad, atol=1e-10, rtol=1e-10)


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_weights_under_dropout_are_those_the_output_used(dt):
    """Under dropout the returned per-head weights are P * keep / (1 - p) with the forward's decisions:
    weights @ v reproduces the attention output exactly as the kernels formed it."""
    import torch

    from gguf_train_b200 import functional as Fn

    O.manual_seed(9)
    B, H, L, D, p, seed = 1, 2, 80, 64, 0.3, 4242
    q, k, v = (seeded((B, H, L, D), dt, 0.5) for _ in range(3))
    tq, tk, tv = (to_dev(x, dt) for x in (q, k, v))
    out, lse = Fn.sdpa_forward(tq, tk, tv, None, None, True, dropout_p=p, seed=seed)
    w = Fn.attention_weights(tq, tk, lse, None, None, True, average=False, dropout_p=p, seed=seed)
    tol = 1e-5 if dt == "f32" else 2e-2  # 16-bit: the weights and the output are each rounded to bf16
    torch.testing.assert_close(torch.matmul(w.float(), tv.float()), out.float(), atol=tol, rtol=tol)
    frac = float((w == 0)[0, :, -1].float().mean())  # the last row sees every key: ~30% dropped
    assert 0.15 < frac < 0.45
