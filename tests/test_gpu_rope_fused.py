"""Prefill attention with RoPE fused in (gtb_sdpa_fwd_rope / functional.sdpa_forward_rope): the
reference applies gt_rope to q and k (csrc/gt_ops_nn.cpp:2409-2421) and then gt_flash_attention
(csrc/gt_ops_nn.cpp:2423-2525). On the tcgen05 kernel q is rotated in shared memory inside the
kernel from a (cos, sin) table of its positions and k once into k_rot; the results must equal
rope() on q and k followed by sdpa_forward bit for bit (both already pinned to the oracle), and the
oracle's rope + attention within the 16-bit tolerance."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, seeded, to_dev

pytestmark = pytest.mark.gpu


def _dt(name):
    import torch

    return {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[name]


@pytest.mark.parametrize("dtype,B,H,Hkv,L,D,n_dims,mode,causal,pos_kind", [
    ("bf16", 2, 8, 2, 300, 128, 128, 0, True, "arange"),     # ragged last tile, GQA, normal pairs
    ("bf16", 1, 4, 4, 512, 128, 64, 2, True, "offset"),      # NeoX, partial rotation, positions from 1000
    ("f16", 2, 4, 1, 257, 64, 64, 2, False, "scattered"),    # head size 64, NeoX, scattered positions
    ("f16", 1, 2, 2, 384, 64, 32, 0, True, "arange"),        # normal pairs over half the head
    ("bf16", 1, 2, 1, 8448, 64, 64, 0, True, "arange"),      # 33 tile pairs: the one-CTA-per-item launch
])
def test_fused_rope_equals_rope_then_attention(dtype, B, H, Hkv, L, D, n_dims, mode, causal, pos_kind):
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    dt = _dt(dtype)
    g = torch.Generator(device="cuda")
    g.manual_seed(L + D)
    q = (torch.randn((B, H, L, D), generator=g, device="cuda") * 0.5).to(dt)
    k = (torch.randn((B, Hkv, L, D), generator=g, device="cuda") * 0.5).to(dt)
    v = (torch.randn((B, Hkv, L, D), generator=g, device="cuda") * 0.5).to(dt)
    if pos_kind == "arange":
        pos = torch.arange(L, dtype=torch.int32, device="cuda")
    elif pos_kind == "offset":
        pos = torch.arange(1000, 1000 + L, dtype=torch.int32, device="cuda")
    else:
        pos = torch.tensor((np.arange(L) * 131 + 7) % 9000, dtype=torch.int32, device="cuda")
    out, lse, k_rot = Fn.sdpa_forward_rope(q, k, v, pos, n_dims, mode, 10000.0, 1.0, is_causal=causal,
                                           q_in_kernel=True)
    assert _C.last_path() == "tcgen05+rope"
    assert _C.device_status() == 0
    out2, lse2, k_rot2 = Fn.sdpa_forward_rope(q, k, v, pos, n_dims, mode, 10000.0, 1.0, is_causal=causal)
    assert _C.last_path() == "tcgen05"  # the default: q rotated in HBM first
    qr = gtb.rope(q, pos, n_dims, mode, 0, 10000.0, 1.0)
    kr = gtb.rope(k, pos, n_dims, mode, 0, 10000.0, 1.0)
    want_out, want_lse = Fn.sdpa_forward(qr, kr, v, None, None, causal)
    assert _C.last_path() == "tcgen05"
    assert torch.equal(k_rot, kr)
    assert torch.equal(out, want_out)
    assert torch.equal(lse, want_lse)
    assert torch.equal(k_rot2, kr) and torch.equal(out2, want_out) and torch.equal(lse2, want_lse)


def test_fused_rope_matches_the_oracle():
    """Against the oracle's restatement of ggml's rope followed by its attention (bf16 inputs, the
    16-bit tolerance 2e-2 / 1e-2): rope rounded to bf16 as the reference's bf16 tensors would be."""
    import torch

    from gguf_train_b200 import functional as Fn

    B, H, Hkv, L, D = 1, 4, 2, 200, 128
    O.manual_seed(5)
    q, k, v = seeded((B, H, L, D), "bf16", 0.5), seeded((B, Hkv, L, D), "bf16", 0.5), seeded((B, Hkv, L, D), "bf16", 0.5)
    pos = np.arange(L) + 17
    out, _, k_rot = Fn.sdpa_forward_rope(to_dev(q, "bf16"), to_dev(k, "bf16"), to_dev(v, "bf16"),
                                         torch.tensor(pos, dtype=torch.int32).cuda(), 128, 0, 10000.0, 1.0,
                                         is_causal=True, q_in_kernel=True)
    qr = O.round_to(O.rope(q, pos, 128, 0, 10000.0, 1.0), O.BF16)
    kr = O.round_to(O.rope(k, pos, 128, 0, 10000.0, 1.0), O.BF16)
    assert_close(k_rot, kr, 2e-2, 1e-2, "k_rot")
    want = O.sdpa_fwd(qr, kr, v, is_causal=True)
    assert_close(out, want, 2e-2, 1e-2, "fused rope attention")


def test_fused_rope_falls_back_where_the_kernel_does_not_rotate():
    """A mask (or an fp32 q) takes the unfused route inside the same call: q rotated into a scratch
    copy, then the forward; the results still equal rope then attention."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    B, H, L, D = 2, 4, 160, 64
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    for dt in (torch.bfloat16, torch.float32):
        q, k, v = ((torch.randn((B, H, L, D), generator=g, device="cuda") * 0.5).to(dt) for _ in range(3))
        mask = torch.ones((B, 1, 1, L), dtype=torch.bool, device="cuda")
        mask[..., L - 9:] = False
        pos = torch.arange(L, dtype=torch.int32, device="cuda")
        out, lse, k_rot = Fn.sdpa_forward_rope(q, k, v, pos, D, 2, 10000.0, 1.0, mask=mask, q_in_kernel=True)
        assert _C.last_path() != "tcgen05+rope"
        qr = gtb.rope(q, pos, D, 2, 0, 10000.0, 1.0)
        kr = gtb.rope(k, pos, D, 2, 0, 10000.0, 1.0)
        want_out, want_lse = Fn.sdpa_forward(qr, kr, v, mask)
        assert torch.equal(k_rot, kr)
        assert torch.equal(out, want_out)
        assert torch.equal(lse, want_lse)


def test_fused_rope_rejects_bad_positions():
    import torch

    from gguf_train_b200 import functional as Fn

    q = torch.zeros((1, 2, 64, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(RuntimeError, match="pos"):
        Fn.sdpa_forward_rope(q, q, q, torch.arange(10, dtype=torch.int32, device="cuda"), 64)
    with pytest.raises(RuntimeError, match="int32"):
        Fn.sdpa_forward_rope(q, q, q, torch.arange(64, device="cuda"), 64)
