"""Dropout on the attention probabilities inside the kernels, against a float64 reference.

The reference's dropout path (gguf_train/nn/functional.py:750-767) is inverted dropout on the
softmax probabilities: out = (P * Z) v with Z = keep / (1 - p). Its gradients (the composite's
autograd) are dv = (P * Z)^T dO, dP = Z * (dO v^T), dS = P * (dP - rowsum(dO * out)), dq = scale dS k,
dk = scale dS^T q, summed over the query heads of a kv head. The engine's keep decisions are a
counter-based hash of (seed, batch * heads + head, query, key), restated here in numpy from its
published definition (lowbias32, Chris Wellons, 2018), so the reference uses exactly the kernels'
mask. Cases cover the tcgen05 kernels (bf16/f16, D 64/128, causal, GQA, a key-padding mask, the
fused and the deterministic dq) and the SIMT kernels (f32)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, seeded, to_dev

pytestmark = pytest.mark.gpu

M32 = np.uint64(0xFFFFFFFF)


def _h32(x):
    x = np.asarray(x, dtype=np.uint64) & M32
    x ^= x >> np.uint64(16)
    x = (x * np.uint64(0x7FEB352D)) & M32
    x ^= x >> np.uint64(15)
    x = (x * np.uint64(0x846CA68B)) & M32
    x ^= x >> np.uint64(16)
    return x


def keep_mask(seed: int, p: float, B: int, H: int, L: int, S: int) -> np.ndarray:
    """keep[b, h, l, s] of the engine's dropout with this seed and probability."""
    thr = np.uint64(min(int(np.float64(np.float32(p)) * 4294967296.0), 0xFFFFFFFF))
    lo, hi = np.uint64(seed & 0xFFFFFFFF), np.uint64((seed >> 32) & 0xFFFFFFFF)
    bh = np.arange(B * H, dtype=np.uint64)
    head = _h32(hi ^ _h32(lo ^ bh))                                   # (B*H,)
    row = _h32(head[:, None] ^ np.arange(L, dtype=np.uint64)[None])   # (B*H, L)
    x = _h32((row[:, :, None] + np.arange(S, dtype=np.uint64)[None, None]) & M32)
    return (x >= thr).reshape(B, H, L, S)


def reference(q, k, v, g, mask, is_bool, scale, causal, keep, p):
    """float64 out, dq, dk, dv of attention with inverted dropout (mask `keep`)."""
    B, H, L, D = q.shape
    Hkv, S = k.shape[1], k.shape[2]
    G = H // Hkv
    ke, ve = np.repeat(k, G, axis=1), np.repeat(v, G, axis=1)
    s = np.einsum("bhld,bhsd->bhls", q, ke) * scale
    if causal:
        s = s + np.where(np.arange(S)[None, :] > np.arange(L)[:, None], -np.inf, 0.0)
    if mask is not None:
        m = np.broadcast_to(mask, (B, H, L, S))
        s = np.where(m == 0, -np.inf, s) if is_bool else s + m
    mx = s.max(-1, keepdims=True)
    P = np.exp(s - mx)
    P /= P.sum(-1, keepdims=True)
    Z = keep / (1.0 - float(np.float32(p)))
    out = np.einsum("bhls,bhsd->bhld", P * Z, ve)
    dP = np.einsum("bhld,bhsd->bhls", g, ve) * Z
    dS = P * (dP - (g * out).sum(-1, keepdims=True))
    dq = np.einsum("bhls,bhsd->bhld", dS, ke) * scale
    dk = np.einsum("bhls,bhld->bhsd", dS, q).reshape(B, Hkv, G, S, D).sum(2) * scale
    dv = np.einsum("bhls,bhld->bhsd", P * Z, g).reshape(B, Hkv, G, S, -1).sum(2)
    return out, dq, dk, dv


CASES = [
    # dtype, B, H, Hkv, L, S, D, causal, p, mask kind, tolerance (abs, rel)
    ("bf16", 1, 4, 2, 200, 200, 128, True, 0.3, None, (2e-2, 1e-2)),     # tcgen05, fused dq
    ("bf16", 2, 2, 1, 130, 260, 128, False, 0.1, None, (2e-2, 1e-2)),
    ("f16", 1, 4, 4, 130, 190, 64, False, 0.5, "kpm", (2e-2, 1e-2)),     # tcgen05 mask + dropout, D = 64
    ("f32", 1, 4, 2, 70, 90, 64, True, 0.2, None, (1e-4, 1e-4)),         # SIMT
    ("f32", 2, 2, 2, 33, 47, 16, False, 0.4, "kpm", (1e-4, 1e-4)),       # SIMT with a mask
]


@pytest.mark.parametrize("dt,B,H,Hkv,L,S,D,causal,p,kind,tol", CASES)
def test_dropout_forward_backward_match_the_reference(dt, B, H, Hkv, L, S, D, causal, p, kind, tol):
    import torch

    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    O.manual_seed(L + S + D)
    sc = 0.5 if dt in ("bf16", "f16") else 1.0
    q, k, v = seeded((B, H, L, D), dt, sc), seeded((B, Hkv, S, D), dt, sc), seeded((B, Hkv, S, D), dt, sc)
    g = seeded((B, H, L, D), dt)
    mask = mt = None
    if kind == "kpm":
        mask = np.ones((B, 1, 1, S))
        mask[..., S - 20:] = 0
        mt = torch.tensor(mask != 0).cuda()
    seed = 0x1234_5678_9ABC + L
    scale = D ** -0.5
    tq, tk, tv = (to_dev(x, dt) for x in (q, k, v))
    out, lse = Fn.sdpa_forward(tq, tk, tv, mt, scale, causal, dropout_p=p, seed=seed)
    path = _C.last_path()
    keep = keep_mask(seed, p, B, H, L, S)
    want = reference(q, k, v, g, mask, True, float(np.float32(scale)), causal, keep, p)
    assert_close(out, want[0], *tol, f"dropout forward ({path})")
    for det in (False, True):
        grads = Fn.sdpa_backward(to_dev(g, dt), tq, tk, tv, mt, out, lse, scale, causal, deterministic=det,
                                 dropout_p=p, seed=seed)
        torch.cuda.synchronize()
        assert _C.device_status() == 0
        for name, got, w in zip(("dq", "dk", "dv"), grads, want[1:]):
            assert_close(got, w, *tol, f"dropout {name} ({_C.last_path()}, deterministic={det})")
    if dt in ("bf16", "f16"):
        assert path == "tcgen05"


def test_dropout_keeps_the_stated_fraction_and_repeats_per_seed():
    """With q = 0 every allowed key has weight 1/S and v = 1, so each output element is the kept
    fraction of its row divided by (1 - p): its mean over many rows is 1. The same seed repeats
    exactly; another seed gives another mask."""
    import torch

    from gguf_train_b200 import functional as Fn

    B, H, L, S, D, p = 2, 8, 512, 512, 128, 0.3
    q = torch.zeros((B, H, L, D), dtype=torch.bfloat16, device="cuda")
    k = torch.randn((B, H, S, D), device="cuda").to(torch.bfloat16)
    v = torch.ones((B, H, S, D), dtype=torch.bfloat16, device="cuda")
    a, _ = Fn.sdpa_forward(q, k, v, None, None, False, dropout_p=p, seed=7)
    b, _ = Fn.sdpa_forward(q, k, v, None, None, False, dropout_p=p, seed=7)
    c, _ = Fn.sdpa_forward(q, k, v, None, None, False, dropout_p=p, seed=8)
    assert torch.equal(a, b) and not torch.equal(a, c)
    rows = a[..., 0].float()
    # each row: (kept of 512) / 512 / 0.7; over 8192 rows the mean's standard error is ~1.4e-3
    assert abs(float(rows.mean()) - 1.0) < 0.01
    assert 0.8 < float(rows.std()) / (np.sqrt(p * (1 - p) / S) / (1 - p)) < 1.2


def test_sdpa_dropout_through_autograd_follows_torch_manual_seed():
    """scaled_dot_product_attention(dropout_p > 0) draws its seed from torch's generator: after the
    same torch.manual_seed the call repeats, and its gradients are the reference's for that seed."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import functional as Fn

    O.manual_seed(4)
    B, H, L, D, p = 1, 2, 96, 64, 0.25
    q, k, v = (seeded((B, H, L, D), "bf16", 0.5) for _ in range(3))
    g = seeded((B, H, L, D), "bf16")
    torch.manual_seed(123)
    seed = Fn.dropout_seed()
    outs = []
    for _ in range(2):
        torch.manual_seed(123)
        tq, tk, tv = (to_dev(x, "bf16", True) for x in (q, k, v))
        o = gtb.scaled_dot_product_attention(tq, tk, tv, dropout_p=p, is_causal=True)
        o.backward(to_dev(g, "bf16"))
        outs.append((o.detach(), tq.grad, tk.grad, tv.grad))
    assert torch.equal(outs[0][0], outs[1][0])
    want = reference(q, k, v, g, None, True, float(np.float32(D ** -0.5)), True, keep_mask(seed, p, B, H, L, L), p)
    for got, w, name in zip(outs[0], want, ("out", "dq", "dk", "dv")):
        assert_close(got, w, 2e-2, 1e-2, f"sdpa dropout {name}")
