"""The tensor-core linear layer (gtb_linear, the role of the reference's gt_linear,
csrc/gt_ops_nn.cpp:256-335): c = a b^T + bias for bf16/f16 against a float64 product of the same
16-bit values, forward and autograd backward, at shapes with ragged tile edges; and the bf16
MultiheadAttention whose projections run on it."""

from __future__ import annotations

import numpy as np
import pytest

from tests._util import assert_close

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("dt,M,N,K,bias", [
    ("bf16", 512, 1536, 512, True),     # MHA in-projection of 512 tokens
    ("bf16", 300, 200, 136, True),      # ragged M, N (two N tiles of 128 would not fit: BN = 256), K tail
    ("f16", 129, 64, 8, False),         # one K step, N < 128
    ("bf16", 1000, 264, 1000, True),    # N just past 256: a second N tile
])
def test_linear_matches_a_float64_product(dt, M, N, K, bias):
    import torch

    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    tdt = {"bf16": torch.bfloat16, "f16": torch.float16}[dt]
    g = torch.Generator(device="cuda")
    g.manual_seed(M + N + K)
    a = torch.randn((M, K), generator=g, device="cuda").to(tdt)
    b = (torch.randn((N, K), generator=g, device="cuda") / K ** 0.5).to(tdt)
    bb = torch.randn((N,), generator=g, device="cuda").to(tdt) if bias else None
    c = Fn._linear_2d(a, b, bb)
    torch.cuda.synchronize()
    assert _C.device_status() == 0
    want = a.double().cpu().numpy() @ b.double().cpu().numpy().T
    if bias:
        want = want + bb.double().cpu().numpy()
    assert_close(c, want, 2e-2, 1e-2, f"linear {dt} {M}x{N}x{K}")


def test_linear_autograd_matches_torch():
    import torch

    from gguf_train_b200 import functional as Fn

    torch.manual_seed(0)
    x = torch.randn((4, 96, 256), device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = (torch.randn((384, 256), device="cuda") / 16).to(torch.bfloat16).requires_grad_()
    b = torch.randn((384,), device="cuda", dtype=torch.bfloat16, requires_grad=True)
    gy = torch.randn((4, 96, 384), device="cuda", dtype=torch.bfloat16)
    y = Fn.linear(x, w, b)
    y.backward(gy)
    xd, wd, bd = (t.detach().double().requires_grad_() for t in (x, w, b))
    yd = torch.nn.functional.linear(xd, wd, bd)
    yd.backward(gy.double())
    for got, want, name in ((y, yd, "y"), (x.grad, xd.grad, "dx"), (w.grad, wd.grad, "dw"), (b.grad, bd.grad, "db")):
        assert_close(got, want.detach().cpu().numpy(), 2e-2 * max(1.0, float(want.abs().max()) / 8), 1e-2, name)


def test_bf16_mha_projections_on_the_repo_gemm():
    """A bf16 MultiheadAttention (self-attention, packed weights, key padding): output and input
    gradient against the same module in float64 (torch's own ops) within bf16 tolerance."""
    import torch

    import gguf_train_b200 as gtb

    torch.manual_seed(3)
    E, H, B, L = 256, 4, 2, 192
    m = gtb.MultiheadAttention(E, H, batch_first=True, device="cuda", dtype=torch.bfloat16)
    with torch.no_grad():
        m.in_proj_bias.normal_(0, 0.1)
    x = torch.randn((B, L, E), device="cuda").to(torch.bfloat16).requires_grad_()
    kpm = torch.zeros((B, L), dtype=torch.bool, device="cuda")
    kpm[1, -30:] = True
    y, _ = m(x, x, x, key_padding_mask=kpm, need_weights=False)
    y.float().sum().backward()
    # float64 reference of the same module, with torch ops throughout
    xd = x.detach().double().requires_grad_()
    W, bi = m.in_proj_weight.detach().double(), m.in_proj_bias.detach().double()
    q, k, v = (torch.nn.functional.linear(xd, w_, b_).view(B, L, H, E // H).transpose(1, 2)
               for w_, b_ in zip(W.chunk(3), bi.chunk(3)))
    s = q @ k.transpose(-1, -2) * (E // H) ** -0.5 + torch.where(kpm, -1e9, 0.0).double()[:, None, None, :]
    o = (torch.softmax(s, -1) @ v).transpose(1, 2).reshape(B, L, E)
    yd = torch.nn.functional.linear(o, m.out_proj.weight.detach().double(), m.out_proj.bias.detach().double())
    yd.sum().backward()
    assert_close(y, yd.detach().cpu().numpy(), 3e-2, 2e-2, "bf16 MHA output")
    assert_close(x.grad, xd.grad.cpu().numpy(), 5e-2, 3e-2, "bf16 MHA dx")
