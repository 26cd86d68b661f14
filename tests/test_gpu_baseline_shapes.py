"""Parity at the benchmarked shapes: each GPU workload that bench.py times runs here at its full size,
and sampled (batch, head) slices are compared with the CPU oracle (the restatement of
gt_flash_attention, csrc/gt_ops_nn.cpp:2423-2525, and of FlashAttentionFn.backward,
gguf_train/_functions.py:1934-1965). Heads and kv-head groups are independent, so a slice checked
at full length is checked exactly as it ran inside the full launch.

Inputs are generated on the device from a seeded torch generator with the configurations'
distributions (q, k, v ~ N(0,1)*0.5, upstream gradient N(0,1)), like the bench; the sampled slices
are copied back for the oracle. Tolerance 2e-2 abs / 1e-2 rel (bf16/f16, the north star's)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-2, 1e-2


def _inputs(B, H, Hkv, L, D, seed, grad=False):
    import torch

    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = (torch.randn((B, H, L, D), generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    k = (torch.randn((B, Hkv, L, D), generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    v = (torch.randn((B, Hkv, L, D), generator=g, device="cuda") * 0.5).to(torch.bfloat16)
    do = torch.randn((B, H, L, D), generator=g, device="cuda").to(torch.bfloat16) if grad else None
    return q, k, v, do


def _host(t):
    return t.detach().double().cpu().numpy()


def _lse_rows(q, k, rows, scale):
    """float64 log-sum-exp of causal scores for the given query rows of one head."""
    s = (q[rows] @ k.T) * scale
    s[np.arange(k.shape[0])[None, :] > rows[:, None]] = -np.inf
    mx = s.max(axis=1, keepdims=True)
    return (mx + np.log(np.exp(s - mx).sum(axis=1, keepdims=True)))[:, 0]


def test_config3_prefill_full_size():
    """Config 3: causal GQA prefill, B=8 Hq=32 Hkv=8 L=S=4096 D=128 bf16 (the bench's default line):
    output and lse of three (batch, head) slices, the last head of the last sequence included."""
    import torch

    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    B, H, Hkv, L, D = 8, 32, 8, 4096, 128
    q, k, v, _ = _inputs(B, H, Hkv, L, D, 1234)
    scale = 1.0 / np.sqrt(D)
    out, lse = Fn.sdpa_forward(q, k, v, None, scale, True, need_lse=True)
    torch.cuda.synchronize()
    assert _C.device_status() == 0
    sc32 = float(np.float32(scale))
    for b, h in ((0, 0), (3, 17), (7, 31)):
        hk = h // (H // Hkv)
        qs, ks, vs = _host(q[b:b + 1, h:h + 1]), _host(k[b:b + 1, hk:hk + 1]), _host(v[b:b + 1, hk:hk + 1])
        want = O.sdpa_fwd(qs, ks, vs, scale=sc32, is_causal=True)
        assert_close(out[b:b + 1, h:h + 1], want, ATOL, RTOL, f"config 3 out (b={b}, h={h})")
        rows = np.array([0, 1, 2047, 3333, L - 1])
        assert_close(lse[b, h, rows], _lse_rows(qs[0, 0], ks[0, 0], rows, sc32), 1e-3, 1e-4,
                     f"config 3 lse (b={b}, h={h})")


def test_config4_training_step_full_size():
    """Config 4: causal GQA forward + backward, B=4 Hq=32 Hkv=8 L=S=8192 D=128 bf16. dq, dk, dv of two
    (batch, kv head) groups (all four query heads of each, every row and key) against the oracle's
    backward, for the default backward (dq summed with f32 reductions inside the dK/dV kernel, over
    64 key blocks per query row here) and for the deterministic one (separate dq kernel); the
    forward output of one head per group too."""
    import torch

    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    B, H, Hkv, L, D = 4, 32, 8, 8192, 128
    G = H // Hkv
    q, k, v, do = _inputs(B, H, Hkv, L, D, 4321, grad=True)
    scale = 1.0 / np.sqrt(D)
    out, lse = Fn.sdpa_forward(q, k, v, None, scale, True, need_lse=True)
    grads = {det: Fn.sdpa_backward(do, q, k, v, None, out, lse, scale, True, deterministic=det)
             for det in (False, True)}
    torch.cuda.synchronize()
    assert _C.device_status() == 0
    groups = ((0, 0), (3, 7))  # (batch, kv head): the first and the last
    qs = np.concatenate([_host(q[b:b + 1, hk * G:(hk + 1) * G]) for b, hk in groups])
    ks = np.concatenate([_host(k[b:b + 1, hk:hk + 1]) for b, hk in groups])
    vs = np.concatenate([_host(v[b:b + 1, hk:hk + 1]) for b, hk in groups])
    gs = np.concatenate([_host(do[b:b + 1, hk * G:(hk + 1) * G]) for b, hk in groups])
    sc32 = float(np.float32(scale))
    dq, dk, dv = O.sdpa_bwd(qs, ks, vs, gs, scale=sc32, is_causal=True)
    for i, (b, hk) in enumerate(groups):
        h = hk * G + (i % G)
        want = O.sdpa_fwd(qs[i:i + 1, i % G:i % G + 1], ks[i:i + 1], vs[i:i + 1], scale=sc32, is_causal=True)
        assert_close(out[b:b + 1, h:h + 1], want, ATOL, RTOL, f"config 4 out (b={b}, h={h})")
        for det, (gq, gk, gv) in grads.items():
            what = f"config 4 (b={b}, kv head {hk}, {'deterministic' if det else 'fused'} dq)"
            assert_close(gq[b:b + 1, hk * G:(hk + 1) * G], dq[i:i + 1], ATOL, RTOL, "dq " + what)
            assert_close(gk[b:b + 1, hk:hk + 1], dk[i:i + 1], ATOL, RTOL, "dk " + what)
            assert_close(gv[b:b + 1, hk:hk + 1], dv[i:i + 1], ATOL, RTOL, "dv " + what)
    # the deterministic backward repeats bit for bit
    again = Fn.sdpa_backward(do, q, k, v, None, out, lse, scale, True, deterministic=True)
    for a, b2 in zip(again, grads[True]):
        assert torch.equal(a, b2)


def test_config5a_decode_full_size():
    """Config 5a: one decode step of B=64 sequences (Hq=32, Hkv=8, D=128, f16 q) against Q8_0 caches of
    Smax=32768 rows with lengths uniform in [1024, 32768], as the bench runs it (the persistent
    tensor-core kernel, in-kernel plan for <= 256 sequences, split-KV chunks and the combine): four
    sequences, the longest included, against the oracle (dequantise, then gt_flash_attention)."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    B, H, Hkv, D, Smax = 64, 32, 8, 128, 32768
    g = torch.Generator(device="cuda")
    g.manual_seed(77)
    lens = torch.randint(1024, Smax + 1, (B,), generator=g, device="cuda").to(torch.int32)
    row = D // 32 * 34
    kq = torch.empty((B, Hkv, Smax, row), dtype=torch.uint8, device="cuda")
    vq = torch.empty_like(kq)
    for b in range(B):
        kq[b] = gtb.quantize_q8_0(torch.randn((Hkv, Smax, D), generator=g, device="cuda"))
        vq[b] = gtb.quantize_q8_0(torch.randn((Hkv, Smax, D), generator=g, device="cuda"))
    q = torch.randn((B, H, 1, D), generator=g, device="cuda").to(torch.float16)
    out = gtb.decode_q8_0(q, kq, vq, lens)
    torch.cuda.synchronize()
    assert _C.device_status() == 0
    ln = lens.cpu().numpy()
    picks = sorted({int(np.argmax(ln)), int(np.argmin(ln)), 0, B - 1})
    for b in picks:
        want = O.decode_q8_0(_host(q[b:b + 1]), kq[b:b + 1].cpu().numpy(), vq[b:b + 1].cpu().numpy(),
                             ln[b:b + 1], Hkv, Smax)
        assert_close(out[b:b + 1], want, ATOL, RTOL, f"config 5a sequence {b} (length {ln[b]})")
    del kq, vq
    torch.cuda.empty_cache()
