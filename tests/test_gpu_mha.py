"""nn.MultiheadAttention (config 2: E=512, H=8, batch_first, L=512, fp32, float mask with -inf at ~10%
plus a key-padding mask of the last 0-64 tokens, need_weights=False) against the float64 oracle
restatement of the reference's MultiheadAttention (transformer.py:70-191), forward and backward,
tolerance 1e-3.

The full B=16 batch runs on the GPU; outputs and input gradients are compared on sampled
sequences (each sequence is independent of the others), weight gradients on a 2-sequence batch
(they sum over the batch)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import mha as M
from oracle import oracle as O
from tests._util import assert_close

pytestmark = pytest.mark.gpu

E, H, L = 512, 8, 512


def _inputs(B, seed):
    O.manual_seed(seed)
    x = O.randn(B, L, E).astype(np.float32).astype(np.float64)
    am = np.where(O.bernoulli(L, L, p=0.1) > 0, -np.inf, 0.0)
    n_pad = (O.rand(B) * 65).astype(np.int64)  # U{0..64}
    kpm = np.zeros((B, L), dtype=bool)
    for b in range(B):
        if n_pad[b]:
            kpm[b, L - n_pad[b]:] = True
    g = O.randn(B, L, E).astype(np.float32).astype(np.float64)
    return x, am, kpm, g


def _module(seed):
    import torch

    import gguf_train_b200 as gtb

    torch.manual_seed(seed)
    m = gtb.MultiheadAttention(E, H, batch_first=True, device="cuda")
    with torch.no_grad():
        m.in_proj_bias.normal_(0, 0.1)
        m.out_proj.bias.normal_(0, 0.1)
    return m


def _run(m, x, am, kpm, g):
    import torch

    tx = torch.tensor(x, dtype=torch.float32, device="cuda", requires_grad=True)
    out, w = m(tx, tx, tx, key_padding_mask=torch.tensor(kpm, device="cuda"),
               attn_mask=torch.tensor(am, dtype=torch.float32, device="cuda"), need_weights=False)
    assert w is None
    m.zero_grad()
    out.backward(torch.tensor(g, dtype=torch.float32, device="cuda"))
    return out, tx.grad


def _weights(m):
    return (m.in_proj_weight.detach().double().cpu().numpy(), m.in_proj_bias.detach().double().cpu().numpy(),
            m.out_proj.weight.detach().double().cpu().numpy(), m.out_proj.bias.detach().double().cpu().numpy())


def test_config2_forward_and_input_grads_on_sampled_sequences():
    from gguf_train_b200 import _C

    B = 16
    x, am, kpm, g = _inputs(B, 2)
    m = _module(2)
    out, dx = _run(m, x, am, kpm, g)
    assert _C.device_status() == 0
    w_in, b_in, w_out, b_out = _weights(m)
    for b in (0, 11):
        sl = slice(b, b + 1)
        want, cache = M.forward(x[sl], x[sl], x[sl], w_in, b_in, w_out, b_out, H, am, kpm[sl])
        assert_close(out[sl], want, 1e-3, 1e-3, f"MHA out, sequence {b}")
        dxq, dxk, dxv, *_ = M.backward(g[sl], cache)
        assert_close(dx[sl], dxq + dxk + dxv, 1e-3, 1e-3, f"MHA dx, sequence {b}")


def test_weight_grads_two_sequences():
    B = 2
    x, am, kpm, g = _inputs(B, 3)
    kpm[1, -40:] = True
    m = _module(3)
    out, dx = _run(m, x, am, kpm, g)
    w_in, b_in, w_out, b_out = _weights(m)
    want, cache = M.forward(x, x, x, w_in, b_in, w_out, b_out, H, am, kpm)
    assert_close(out, want, 1e-3, 1e-3, "MHA out")
    _, _, _, dw_in, db_in, dw_out, db_out = M.backward(g, cache)
    assert_close(m.in_proj_weight.grad, dw_in, 1e-3, 1e-3, "d in_proj_weight")
    assert_close(m.in_proj_bias.grad, db_in, 1e-3, 1e-3, "d in_proj_bias")
    assert_close(m.out_proj.weight.grad, dw_out, 1e-3, 1e-3, "d out_proj.weight")
    assert_close(m.out_proj.bias.grad, db_out, 1e-3, 1e-3, "d out_proj.bias")


def test_true_in_a_bool_attn_mask_blocks_the_position():
    """tests/test_pooling_and_attention.py:262-278 with need_weights=False."""
    import torch

    import gguf_train_b200 as gtb

    torch.manual_seed(2)
    m = gtb.MultiheadAttention(8, 2, batch_first=True, device="cuda").eval()
    x = torch.randn(1, 4, 8, device="cuda")
    causal = torch.triu(torch.ones(4, 4, device="cuda"), diagonal=1).bool()
    out, _ = m(x, x, x, attn_mask=causal, need_weights=False)
    changed = x.clone()
    changed[0, -1] += 5.0
    out2, _ = m(changed, changed, changed, attn_mask=causal, need_weights=False)
    assert (out[0, :-1] - out2[0, :-1]).abs().max().item() < 1e-5
    assert (out[0, -1] - out2[0, -1]).abs().max().item() > 1e-3
