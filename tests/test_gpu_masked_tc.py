"""Masked attention on the tensor-core kernels: forward and backward parity with the oracle.

The reference applies a bool mask (0 = the key may not be attended) or adds a float mask inside its
attention loop (gt_flash_attention, csrc/gt_ops_nn.cpp:2488-2500), with 2-D (L, S) or 4-D masks whose
size-1 dimensions broadcast. These cases run bf16/f16 inputs with D in {64, 128}, the shapes the
tcgen05 kernels take, and assert that they did (gtb_last_path): key-padding masks (B,1,1,S) as
TransformerEncoderLayer passes them, per-head (B,H,L,S) bool masks, additive float masks with -inf
entries in f32/f16/bf16, block-sparse masks whose blocks are wholly masked, a fully masked row,
and a mask viewed through non-contiguous strides. Tolerance 2e-2 abs / 1e-2 rel."""

from __future__ import annotations

import zlib

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, seeded, to_dev

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def _mask(kind, B, H, L, S, rng):
    """(mask values as float64, is_bool): the mask of `kind`, shaped as it is passed."""
    if kind == "kpm":  # key padding: the last n_b keys of sequence b are masked
        m = np.ones((B, 1, 1, S))
        for b in range(B):
            m[b, ..., S - int(rng.integers(0, min(S - 1, 70))):] = 0
        return m, True
    if kind == "bool_bhls":
        m = (rng.random((B, H, L, S)) < 0.75).astype(np.float64)
        m[..., 0] = 1
        return m, True
    if kind == "bool_2d_row":  # (L, S) with one fully masked query row
        m = (rng.random((L, S)) < 0.6).astype(np.float64)
        m[:, 0] = 1
        m[min(5, L - 1)] = 0
        return m, True
    if kind == "float_inf":  # (1,1,L,S) additive with -inf at ~10%
        m = rng.standard_normal((1, 1, L, S)) * 0.5
        drop = rng.random((1, 1, L, S)) < 0.1
        drop[..., 0] = False
        m[drop] = -np.inf
        return m, False
    if kind == "block_sparse":  # (B,1,L,S) bool: a local window in 128-blocks -> whole blocks masked
        lb = np.arange(L)[:, None] // 128
        sb = np.arange(S)[None, :] // 128
        m = (np.abs(lb - sb) <= 1).astype(np.float64)
        return np.broadcast_to(m, (B, 1, L, S)).copy(), True
    if kind == "float_b1l1":  # (B,1,L,1) additive: a per-row constant (softmax-invariant)
        return rng.standard_normal((B, 1, L, 1)), False
    raise ValueError(kind)


def _dev_mask(m, is_bool, mdtype, transposed=False):
    import torch

    if is_bool:
        t = torch.tensor(m != 0).cuda()
    else:
        t = to_dev(O.round_to(m, {"f32": O.F32, "f16": O.F16, "bf16": O.BF16}[mdtype]), mdtype)
    if transposed:  # same values through a non-contiguous view
        t = t.transpose(-1, -2).contiguous().transpose(-1, -2)
    return t


CASES = [
    # dtype, B, H, Hkv, L, S, D, causal, mask kind, float mask dtype, transposed view
    ("bf16", 2, 8, 2, 300, 300, 128, True, "kpm", None, False),
    ("bf16", 2, 4, 4, 200, 333, 128, False, "kpm", None, False),
    ("f16", 1, 4, 2, 256, 256, 64, False, "bool_bhls", None, False),
    ("bf16", 1, 4, 1, 130, 130, 128, True, "bool_2d_row", None, False),
    ("bf16", 2, 4, 2, 257, 190, 128, False, "float_inf", "f32", False),
    ("f16", 1, 2, 2, 384, 384, 64, True, "float_inf", "f16", False),
    ("bf16", 1, 4, 2, 512, 512, 128, False, "float_inf", "bf16", True),
    ("bf16", 2, 4, 2, 640, 640, 128, False, "block_sparse", None, False),
    ("bf16", 2, 2, 1, 200, 200, 64, True, "float_b1l1", "f32", False),
]


@pytest.mark.parametrize("dt,B,H,Hkv,L,S,D,causal,kind,mdt,transposed", CASES)
def test_masked_forward_backward_on_tensor_cores(dt, B, H, Hkv, L, S, D, causal, kind, mdt, transposed):
    import torch

    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    rng = np.random.default_rng(zlib.crc32(f"{kind} {L} {S} {D}".encode()))
    O.manual_seed(int(rng.integers(1 << 30)))
    q, k, v = seeded((B, H, L, D), dt, 0.5), seeded((B, Hkv, S, D), dt, 0.5), seeded((B, Hkv, S, D), dt, 0.5)
    g = seeded((B, H, L, D), dt)
    m, is_bool = _mask(kind, B, H, L, S, rng)
    mt = _dev_mask(m, is_bool, mdt, transposed)
    m_used = m if is_bool else O.round_to(m, {"f32": O.F32, "f16": O.F16, "bf16": O.BF16}[mdt])
    tq, tk, tv = (to_dev(x, dt) for x in (q, k, v))
    scale = D ** -0.5
    out, lse = Fn.sdpa_forward(tq, tk, tv, mt, scale, causal, need_lse=True)
    assert _C.last_path() == "tcgen05", "masked forward did not run on the tensor cores"
    for det in (False, True):
        dq, dk, dv = Fn.sdpa_backward(to_dev(g, dt), tq, tk, tv, mt, out, lse, scale, causal, deterministic=det)
        assert _C.last_path() == "tcgen05", "masked backward did not run on the tensor cores"
        torch.cuda.synchronize()
        assert _C.device_status() == 0
        sc32 = float(np.float32(scale))
        if not det:
            want = O.sdpa_fwd(q, k, v, m_used, is_bool, sc32, causal)
            assert_close(out, want, ATOL, RTOL, f"masked forward {kind}")
        wq, wk, wv = O.sdpa_bwd(q, k, v, g, m_used, is_bool, sc32, causal)
        if kind == "bool_2d_row":
            # the engine's backward gives a fully masked row zero gradients (its forward output is 0);
            # the reference's op-by-op backward would differentiate a softmax over -1e9 scores there
            dead = np.all(m_used == 0, axis=-1)
            wq[:, :, dead] = 0.0
            wk, wv = _without_dead_rows(q, k, v, g, m_used, is_bool, sc32, causal, dead)
        what = f"{kind} ({'deterministic' if det else 'fused'} dq)"
        assert_close(dq, wq, ATOL, RTOL, "dq " + what)
        assert_close(dk, wk, ATOL, RTOL, "dk " + what)
        assert_close(dv, wv, ATOL, RTOL, "dv " + what)


def _without_dead_rows(q, k, v, g, m, is_bool, scale, causal, dead):
    """dk, dv of the oracle backward with the fully masked query rows' upstream gradient set to 0
    (their contribution in the engine, whose forward gives those rows 0)."""
    g2 = g.copy()
    g2[:, :, dead] = 0.0
    _, dk, dv = O.sdpa_bwd(q, k, v, g2, m, is_bool, scale, causal)
    return dk, dv


def test_masked_forward_sdpa_api_key_padding_matches_unmasked_on_the_kept_keys():
    """Through scaled_dot_product_attention: a bool key-padding mask (True = may attend, the
    SDPA convention) gives the same result as slicing the padded keys away."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    O.manual_seed(9)
    B, H, L, S, D, keep = 1, 4, 256, 300, 128, 211
    q, k, v = (to_dev(seeded(s, "bf16", 0.5), "bf16") for s in ((B, H, L, D), (B, H, S, D), (B, H, S, D)))
    mask = torch.zeros((B, 1, 1, S), dtype=torch.bool, device="cuda")
    mask[..., :keep] = True
    got = gtb.scaled_dot_product_attention(q, k, v, attn_mask=mask)
    assert _C.last_path() == "tcgen05"
    want = gtb.scaled_dot_product_attention(q, k[:, :, :keep].contiguous(), v[:, :, :keep].contiguous())
    torch.testing.assert_close(got.float(), want.float(), atol=2e-2, rtol=1e-2)
