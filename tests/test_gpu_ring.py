"""GPU parity of the long-context ring pieces: the log-sum-exp merge kernel against a float64 merge,
and the ring schedule run for 1, 2 and 4 emulated ranks on one GPU (native forward calls on zig-zag
chunks, merged by gtb_attn_merge) against the CPU oracle's causal attention."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close

pytestmark = pytest.mark.gpu


def test_merge_kernel_matches_float64():
    import torch

    from gguf_train_b200 import ring

    g = torch.Generator().manual_seed(3)
    B, H, R, D = 2, 3, 40, 128
    o_acc = torch.randn((B, H, R, D), generator=g, dtype=torch.float64)
    lse_acc = torch.randn((B, H, R), generator=g, dtype=torch.float64) * 3
    o_part = torch.randn((B, H, 2 * R, D), generator=g, dtype=torch.float64)
    lse_part = torch.randn((B, H, 2 * R), generator=g, dtype=torch.float64) * 3
    lse_acc[0, 0, :5] = float("-inf")   # accumulator still empty
    lse_part[0, 1, R:R + 5] = float("-inf")  # part saw no allowed key
    lse_acc[1, 2, 7] = lse_part[1, 2, R + 7] = float("-inf")
    # the second half of a wider partial result (row-range view, as ring_step merges them)
    op, lp = o_part[:, :, R:], lse_part[:, :, R:]
    m = torch.maximum(lse_acc, lp)
    wa = torch.where(lse_acc == float("-inf"), 0.0, torch.exp(lse_acc - m))
    wp = torch.where(lp == float("-inf"), 0.0, torch.exp(lp - m))
    tot = wa + wp
    want_o = torch.where(tot[..., None] > 0, (o_acc * wa[..., None] + op.bfloat16().double() * wp[..., None]) /
                         tot[..., None], o_acc)
    want_l = torch.where(tot > 0, m + torch.log(tot), lse_acc)
    oa, la = o_acc.float().cuda().contiguous(), lse_acc.float().cuda().contiguous()
    part = o_part.bfloat16().cuda()
    lpart = lse_part.float().cuda()
    ring.merge_(oa, la, part[:, :, R:], lpart[:, :, R:])
    torch.cuda.synchronize()
    assert torch.allclose(oa.double().cpu(), want_o, atol=1e-5, rtol=1e-5)
    got_l = la.double().cpu()
    assert torch.equal(torch.isinf(got_l), torch.isinf(want_l))
    fin = ~torch.isinf(want_l)
    assert torch.allclose(got_l[fin], want_l[fin], atol=1e-5, rtol=1e-6)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_emulated_ring_matches_causal_attention(world):
    import torch

    from gguf_train_b200 import ring

    O.manual_seed(11)
    B, H, Hkv, L, D = 1, 4, 2, 1024, 128
    q = O.round_to(O.randn(B, H, L, D) * 0.5, O.BF16)
    k = O.round_to(O.randn(B, Hkv, L, D) * 0.5, O.BF16)
    v = O.round_to(O.randn(B, Hkv, L, D) * 0.5, O.BF16)
    tq, tk, tv = (torch.tensor(x, dtype=torch.float32).cuda().to(torch.bfloat16) for x in (q, k, v))
    got = ring.ring_attention_emulated(tq, tk, tv, world)
    from gguf_train_b200 import _C

    assert _C.device_status() == 0
    assert_close(got, O.sdpa_fwd(q, k, v, is_causal=True), 2e-2, 1e-2, f"ring of {world}")
