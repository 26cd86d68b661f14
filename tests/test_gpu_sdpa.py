"""GPU parity of the attention forward and backward against the CPU oracle.

The oracle restates gt_flash_attention (reference csrc/gt_ops_nn.cpp:2423-2525) and
FlashAttentionFn.backward (gguf_train/_functions.py:1934-1965) in float64. Tolerances: the
north-star's 1e-3 for fp32 (these kernels reach ~1e-6), 2e-2 abs / 1e-2 rel for bf16/fp16,
1e-7 for f64. Inputs come from the reference's generator (mt19937_64 + normal, seed fixed).
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import DT, assert_close, seeded, to_dev

pytestmark = pytest.mark.gpu

# f64: the reference hands the scale to its forward as a C float (gguf_train/_C.py:471) but
# multiplies by the Python double in its backward (_functions.py:1940); the engine uses the float
# value throughout, which moves float64 results by ~1e-8 relative.
TOL = {"f32": (1e-4, 1e-4), "f64": (1e-7, 1e-7), "bf16": (2e-2, 1e-2), "f16": (2e-2, 1e-2)}


def _mask(kind, B, H, L, S, seed):
    """bool: (B,1,L,S), True = may attend, key 0 always allowed; float: (1,1,L,S) additive with
    -inf at ~10% of positions, key 0 finite."""
    if kind is None:
        return None, None
    O.manual_seed(seed)
    if kind == "bool":
        m = O.rand(B, 1, L, S) < 0.7
        m[..., 0] = True
        return m.astype(np.float64), True
    m = O.randn(1, 1, L, S) * 0.5
    drop = O.rand(1, 1, L, S) < 0.1
    drop[..., 0] = False
    m[drop] = -np.inf
    return m, False


def _mask_dev(m, is_bool, dtype):
    import torch

    if m is None:
        return None
    if is_bool:
        return torch.tensor(m != 0).cuda()
    return to_dev(m, dtype)


FWD_CASES = [
    # dtype, B, H, Hkv, L, S, D, Dv, causal, mask
    ("f32", 2, 4, 4, 128, 128, 64, 64, True, None),      # config 1 shape
    ("f32", 2, 3, 3, 4, 5, 6, 6, False, "bool"),        # reference test shape (test_pooling_and_attention.py:349)
    ("f32", 2, 3, 3, 4, 5, 6, 6, False, "float"),
    ("f64", 1, 2, 2, 4, 4, 8, 8, True, None),           # gradcheck shape (test_autograd.py:136)
    ("f32", 2, 4, 2, 96, 128, 64, 64, False, "float"),  # fp32 tiled kernels, mask rows read 4 keys at a time
    ("f32", 1, 2, 2, 100, 132, 64, 64, True, "bool"),
    ("bf16", 1, 4, 2, 300, 300, 128, 128, True, None),  # tcgen05 path, ragged last tile, GQA
    ("bf16", 2, 4, 1, 200, 333, 128, 128, False, None), # tcgen05 path, L != S
    ("bf16", 1, 2, 2, 257, 130, 128, 128, True, None),  # causal with L > S (top-left)
    ("bf16", 1, 2, 2, 100, 700, 128, 128, True, None),  # causal with L < S
    ("f16", 1, 4, 4, 256, 256, 64, 64, True, None),     # tcgen05 path, D = 64, fp16
    ("f16", 2, 2, 1, 64, 1000, 64, 64, False, None),
    ("bf16", 1, 4, 2, 128, 128, 128, 128, False, "float"),  # mask -> SIMT
    ("bf16", 1, 2, 2, 64, 64, 96, 96, True, None),      # D = 96 -> SIMT
    ("f32", 1, 2, 2, 1, 1, 8, 8, True, None),
    ("f32", 1, 2, 2, 3, 0, 8, 8, False, None),          # no keys: output 0
    ("bf16", 1, 1, 1, 1, 1, 128, 128, True, None),
]


@pytest.mark.parametrize("dtype,B,H,Hkv,L,S,D,Dv,causal,mask", FWD_CASES)
def test_forward_matches_oracle(dtype, B, H, Hkv, L, S, D, Dv, causal, mask):
    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    O.manual_seed(1000 + L + S + D)
    sc = 0.5 if dtype in ("bf16", "f16") else 1.0
    q = seeded((B, H, L, D), dtype, sc)
    k = seeded((B, Hkv, S, D), dtype, sc)
    v = seeded((B, Hkv, S, Dv), dtype, sc)
    m, mb = _mask(mask, B, H, L, S, 7)
    if m is not None and not mb:
        m = O.round_to(m, {"f32": O.F32, "f64": O.F64, "bf16": O.BF16, "f16": O.F16}[dtype])
    want = O.sdpa_fwd(q, k, v, m, mb, scale=0.0, is_causal=causal)
    got = gtb.scaled_dot_product_attention(to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype),
                                           attn_mask=_mask_dev(m, mb, dtype), is_causal=causal)
    assert _C.device_status() == 0
    atol, rtol = TOL[dtype]
    assert_close(got, want, atol, rtol, f"forward {dtype} {(B, H, Hkv, L, S, D)} causal={causal} mask={mask}")


@pytest.mark.parametrize("dtype,causal", [("bf16", False), ("f16", False), ("bf16", True)])
def test_forward_rescales_when_the_maximum_jumps_inside_a_block(dtype, causal):
    """Scores that climb along the keys (q . k = A_l * 0.3 s in the first head dimension): rows with
    A_l = 8 see their maximum grow by ~9.8 (log2 units) every 32 keys, so the forward raises its
    exponent offset inside every key block and rescales the probabilities already written; rows with
    A_l in {0, 2, -8} in the same warps never do. Output and lse against the oracle."""
    import gguf_train_b200 as gtb
    from gguf_train_b200 import functional as F
    from gguf_train_b200 import _C

    B, H, Hkv, L, S, D = 1, 2, 1, 256, 384, 128
    O.manual_seed(4242)
    q = O.randn(B, H, L, D) * 0.05
    k = O.randn(B, Hkv, S, D) * 0.05
    v = seeded((B, Hkv, S, D), dtype, 0.5)
    amp = np.array([0.0, 2.0, 8.0, -8.0])[np.arange(L) % 4]
    q[..., 0] = amp
    k[..., 0] = 0.3 * np.arange(S)
    q, k = O.round_to(q, DT[dtype]), O.round_to(k, DT[dtype])
    want = O.sdpa_fwd(q, k, v, None, False, scale=0.0, is_causal=causal)
    sc = np.einsum("bhld,bsd->bhls", q, k[:, 0]) / np.sqrt(D)
    if causal:
        sc = np.where(np.arange(S)[None, :] > np.arange(L)[:, None], -np.inf, sc)
    mx = sc.max(-1, keepdims=True)
    want_lse = (mx + np.log(np.exp(sc - mx).sum(-1, keepdims=True)))[..., 0]
    out, lse = F.sdpa_forward(to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype), None, None, causal)
    assert _C.device_status() == 0
    assert_close(out, want, 2e-2, 1e-2, f"forward {dtype} causal={causal} with climbing scores")
    assert_close(lse, want_lse, 2e-3, 1e-4, "lse with climbing scores")


BWD_CASES = [
    ("f32", 2, 4, 4, 128, 128, 64, 64, True, None),     # config 1: fwd+bwd, tol 1e-3 required
    ("f32", 2, 3, 3, 4, 5, 6, 6, False, "bool"),
    ("f32", 1, 4, 2, 33, 47, 16, 24, False, "float"),
    ("f64", 1, 2, 2, 4, 4, 8, 8, True, None),
    ("f32", 2, 4, 2, 96, 128, 64, 64, False, "float"),  # fp32 tiled kernels, mask rows read 4 keys at a time
    ("f32", 1, 2, 2, 100, 132, 64, 64, True, "bool"),
    ("bf16", 1, 4, 2, 200, 200, 128, 128, True, None),
    ("f16", 1, 2, 2, 130, 70, 64, 64, False, None),
    ("bf16", 1, 4, 1, 384, 384, 128, 128, True, None),   # tcgen05 backward: GQA group of 4, 3 tiles
    ("bf16", 1, 2, 2, 300, 170, 128, 128, True, None),   # causal with L > S
    ("bf16", 1, 2, 1, 150, 400, 128, 128, True, None),   # causal with L < S (key blocks no query sees)
    ("bf16", 2, 2, 2, 256, 256, 64, 64, True, None),     # D = 64
    ("f16", 1, 2, 2, 129, 129, 128, 128, False, None),
]


@pytest.mark.parametrize("dtype,B,H,Hkv,L,S,D,Dv,causal,mask", BWD_CASES)
def test_backward_matches_oracle(dtype, B, H, Hkv, L, S, D, Dv, causal, mask):
    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    O.manual_seed(2000 + L + S + D)
    sc = 0.5 if dtype in ("bf16", "f16") else 1.0
    q = seeded((B, H, L, D), dtype, sc)
    k = seeded((B, Hkv, S, D), dtype, sc)
    v = seeded((B, Hkv, S, Dv), dtype, sc)
    g = seeded((B, H, L, Dv), dtype)
    m, mb = _mask(mask, B, H, L, S, 9)
    dq, dk, dv = O.sdpa_bwd(q, k, v, g, m, mb, is_causal=causal)
    tq, tk, tv = (to_dev(x, dtype, True) for x in (q, k, v))
    out = gtb.scaled_dot_product_attention(tq, tk, tv, attn_mask=_mask_dev(m, mb, dtype), is_causal=causal)
    out.backward(to_dev(g, dtype))
    assert _C.device_status() == 0
    atol, rtol = TOL[dtype]
    if dtype == "f32":
        atol, rtol = 1e-3, 1e-3
    label = f"{dtype} {(B, H, Hkv, L, S, D, Dv)} causal={causal} mask={mask}"
    assert_close(tq.grad, dq, atol, rtol, "dq " + label)
    assert_close(tk.grad, dk, atol, rtol, "dk " + label)
    assert_close(tv.grad, dv, atol, rtol, "dv " + label)


def test_strided_views_give_the_same_result():
    """SDPA on strided views equals SDPA on fresh tensors (reference
    tests/test_views_and_fast_paths.py:334-336): the (B, L, H, D) -> (B, H, L, D) transpose of MHA."""
    import torch

    import gguf_train_b200 as gtb

    O.manual_seed(5)
    B, L, H, D = 2, 160, 4, 128
    base = to_dev(seeded((B, L, 3, H, D), "bf16", 0.5), "bf16")
    q, k, v = (base[:, :, i].transpose(1, 2) for i in range(3))
    got = gtb.scaled_dot_product_attention(q, k, v, is_causal=True)
    want = gtb.scaled_dot_product_attention(q.contiguous(), k.contiguous(), v.contiguous(), is_causal=True)
    assert torch.equal(got, want)


def test_mask_shape_errors():
    """tests/test_pooling_and_attention.py:375-386: bad masks raise 'cannot be broadcast', both via F
    and via FlashAttentionFn.apply directly."""
    import torch

    import gguf_train_b200 as gtb

    q = torch.randn(2, 3, 4, 6, device="cuda")
    k = torch.randn(2, 3, 5, 6, device="cuda")
    v = torch.randn(2, 3, 5, 6, device="cuda")
    for shape in ((2, 3), (4, 6), (7, 4, 5), (2, 3, 4, 5, 1)):
        with pytest.raises(RuntimeError, match="cannot be broadcast"):
            gtb.scaled_dot_product_attention(q, k, v, attn_mask=torch.ones(*shape, dtype=torch.bool, device="cuda"))
    for shape in ((2, 3), (5,), (2, 4, 5)):
        with pytest.raises(RuntimeError, match="cannot be broadcast"):
            gtb.FlashAttentionFn.apply(q, k, v, torch.ones(*shape, dtype=torch.bool, device="cuda"), 0.4, False)
    with pytest.raises(RuntimeError, match="num_heads must be divisible by num_kv_heads"):
        gtb.scaled_dot_product_attention(q, k[:, :2], v[:, :2])
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        gtb.scaled_dot_product_attention(q.cpu(), k.cpu(), v.cpu())


def test_masks_broadcast_from_the_right():
    """tests/test_pooling_and_attention.py:364-373: every right-aligned broadcast of a bool mask
    and its -1e9 additive twin give the composite's answer."""
    import torch

    import gguf_train_b200 as gtb

    O.manual_seed(6)
    q, k, v = seeded((2, 3, 4, 6)), seeded((2, 3, 5, 6)), seeded((2, 3, 5, 6))
    base = O.rand(2, 3, 4, 5) < 0.6
    base[..., 0] = True
    tq, tk, tv = to_dev(q, "f32"), to_dev(k, "f32"), to_dev(v, "f32")
    for mask in (base, base[:, :1], base[:1], base[0], base[0, 0], base[0, 0, :1], base[..., :1, :]):
        m4 = mask.reshape((1,) * (4 - mask.ndim) + mask.shape)
        want = O.sdpa_fwd(q, k, v, np.broadcast_to(m4, (2, 3, 4, 5)).astype(np.float64), True)
        got = gtb.scaled_dot_product_attention(tq, tk, tv, attn_mask=torch.tensor(mask).cuda())
        assert_close(got, want, 1e-5, 1e-5, f"bool mask {mask.shape}")
        additive = torch.zeros(mask.shape).masked_fill(~torch.tensor(mask), -1e9).cuda()
        got = gtb.scaled_dot_product_attention(tq, tk, tv, attn_mask=additive)
        assert_close(got, want, 1e-5, 1e-5, f"additive mask {mask.shape}")


def test_fully_masked_row_gives_zero_output():
    """A row with no allowed key outputs 0 (gt_ops_nn.cpp:2509: inv = 0 when the sum is 0)."""
    import torch

    import gguf_train_b200 as gtb

    q = torch.randn(1, 2, 4, 8, device="cuda")
    k = torch.randn(1, 2, 6, 8, device="cuda")
    v = torch.randn(1, 2, 6, 8, device="cuda")
    mask = torch.ones(4, 6, dtype=torch.bool, device="cuda")
    mask[2] = False
    out = gtb.scaled_dot_product_attention(q, k, v, attn_mask=mask)
    assert torch.all(out[:, :, 2] == 0)
    assert torch.all(out[:, :, 1].abs().sum(-1) > 0)


def test_gradcheck_float64_causal():
    """tests/test_autograd.py:136-140: finite-difference gradcheck of causal SDPA in float64."""
    import torch

    import gguf_train_b200 as gtb

    O.manual_seed(11)
    q, k, v = (to_dev(seeded((1, 2, 4, 8), "f64"), "f64", True) for _ in range(3))
    assert torch.autograd.gradcheck(lambda a, b, c: gtb.scaled_dot_product_attention(a, b, c, is_causal=True), (q, k, v))


def test_backward_sampled_group_at_larger_size():
    """Causal GQA backward at L = S = 1024 (B=2, H=8, Hkv=2): the whole batch on the GPU, one
    (batch, kv head) group checked against the oracle (groups are independent)."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    O.manual_seed(77)
    B, H, Hkv, L, D = 2, 8, 2, 1024, 128
    q = seeded((B, H, L, D), "bf16", 0.5)
    k = seeded((B, Hkv, L, D), "bf16", 0.5)
    v = seeded((B, Hkv, L, D), "bf16", 0.5)
    g = seeded((B, H, L, D), "bf16")
    tq, tk, tv = (to_dev(x, "bf16", True) for x in (q, k, v))
    out = gtb.scaled_dot_product_attention(tq, tk, tv, is_causal=True)
    out.backward(to_dev(g, "bf16"))
    assert _C.device_status() == 0
    b, hk, G = 1, 1, H // Hkv
    hs = slice(hk * G, (hk + 1) * G)
    dq, dk, dv = O.sdpa_bwd(q[b:b + 1, hs], k[b:b + 1, hk:hk + 1], v[b:b + 1, hk:hk + 1], g[b:b + 1, hs], is_causal=True)
    assert_close(tq.grad[b:b + 1, hs], dq, 2e-2, 1e-2, "dq sampled group")
    assert_close(tk.grad[b:b + 1, hk:hk + 1], dk, 2e-2, 1e-2, "dk sampled group")
    assert_close(tv.grad[b:b + 1, hk:hk + 1], dv, 2e-2, 1e-2, "dv sampled group")
    del torch


def test_forward_persistent_ctas_over_many_items():
    """Causal GQA bf16 forward with more work items (pairs of 128-row query tiles x heads x batch) than
    SMs, so that each persistent CTA of the tcgen05 kernel runs several items in a row and its K/V
    ring, barrier phases and TMEM carry over between them: B=4, H=16, Hkv=4, L=S=2048 is 512 items
    for 148 CTAs. Three (batch, head) slices checked against the oracle at full length, the lse too."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C
    from gguf_train_b200 import functional as Fn

    O.manual_seed(21)
    B, H, Hkv, L, D = 4, 16, 4, 2048, 128
    q = seeded((B, H, L, D), "bf16", 0.5)
    k = seeded((B, Hkv, L, D), "bf16", 0.5)
    v = seeded((B, Hkv, L, D), "bf16", 0.5)
    tq, tk, tv = (to_dev(x, "bf16") for x in (q, k, v))
    out, lse = Fn.sdpa_forward(tq, tk, tv, None, D ** -0.5, True, need_lse=True)
    torch.cuda.synchronize()
    assert _C.device_status() == 0
    G = H // Hkv
    for b, h in ((0, 0), (2, 6), (3, 15)):
        hk = h // G
        want = O.sdpa_fwd(q[b:b + 1, h:h + 1], k[b:b + 1, hk:hk + 1], v[b:b + 1, hk:hk + 1], is_causal=True)
        assert_close(out[b:b + 1, h:h + 1], want, *TOL["bf16"], f"out (b={b}, h={h})")
        # lse = log sum_k exp(scale * q.k) over the allowed keys, from a float64 restatement
        qf, kf = q[b, h].astype(np.float64), k[b, hk].astype(np.float64)
        rows = np.array([0, 1, 777, L - 1])
        s = (qf[rows] @ kf.T) * float(np.float32(D ** -0.5))
        s[np.arange(L)[None, :] > rows[:, None]] = -np.inf
        mx = s.max(axis=1, keepdims=True)
        want_lse = (mx + np.log(np.exp(s - mx).sum(axis=1, keepdims=True)))[:, 0]
        assert_close(lse[b, h, rows], want_lse, 1e-3, 1e-4, f"lse (b={b}, h={h})")


def test_forward_just_past_the_persistent_limit():
    """L = S = 8448 (33 tile pairs) is one CTA per item in blockIdx order, the mode used for
    sequences longer than 8192 rows; the last 256 query rows of one head checked against the
    oracle's row-range forward (causal masking uses absolute rows)."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    O.manual_seed(22)
    B, H, Hkv, L, D = 1, 4, 2, 8448, 128
    q = seeded((B, H, L, D), "bf16", 0.5)
    k = seeded((B, Hkv, L, D), "bf16", 0.5)
    v = seeded((B, Hkv, L, D), "bf16", 0.5)
    out = gtb.scaled_dot_product_attention(*(to_dev(x, "bf16") for x in (q, k, v)), is_causal=True)
    torch.cuda.synchronize()
    assert _C.device_status() == 0
    h, hk, off = 3, 1, L - 256
    want = O.sdpa_fwd_reforder(q[:, h:h + 1, off:], k[:, hk:hk + 1], v[:, hk:hk + 1], float(np.float32(D ** -0.5)),
                               True, 0, off)
    assert_close(out[:, h:h + 1, off:], want, *TOL["bf16"], "out, last 256 rows of head 3")


_SPLIT_SCRIPT = r"""
import sys
import numpy as np
sys.path.insert(0, {root!r})
from oracle import oracle as O
from tests._util import seeded, to_dev
import gguf_train_b200 as gtb
from gguf_train_b200 import _C
O.manual_seed(4242)
B, H, Hkv, L, D = 1, 4, 1, 384, 128
q = seeded((B, H, L, D), "bf16", 0.5)
k = seeded((B, Hkv, L, D), "bf16", 0.5)
v = seeded((B, Hkv, L, D), "bf16", 0.5)
g = seeded((B, H, L, D), "bf16")
want = O.sdpa_bwd(q, k, v, g, None, None, is_causal=True)
tq, tk, tv = (to_dev(x, "bf16", True) for x in (q, k, v))
gtb.scaled_dot_product_attention(tq, tk, tv, is_causal=True).backward(to_dev(g, "bf16"))
assert _C.device_status() == 0
for name, got, ref in zip(("dq", "dk", "dv"), (tq.grad, tk.grad, tv.grad), want):
    err = np.abs(got.float().cpu().numpy() - ref)
    assert np.all(err <= 2e-2 + 1e-2 * np.abs(ref)), (name, float(err.max()))
print("SPLIT-OK")
"""


def test_backward_split_dq_kernel_matches_oracle():
    """GTB_BWD_SPLIT_DQ=1 selects the separate (deterministic) dQ kernel instead of the dQ sums
    inside the dK/dV kernel; the variable is read once per process, so the check runs in a child."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ, GTB_BWD_SPLIT_DQ="1")
    r = subprocess.run([sys.executable, "-c", _SPLIT_SCRIPT.format(root=root)], env=env, cwd=root,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "SPLIT-OK" in r.stdout, r.stdout + r.stderr


def test_backward_fused_dq_repeats_within_rounding():
    """The fused dQ adds f32 partial sums in whatever order the CTAs reach L2: two runs of the same
    backward agree to f32 rounding of the sums (well inside the bf16 output's ulp), dK and dV exactly."""
    import torch

    import gguf_train_b200 as gtb

    O.manual_seed(99)
    B, H, Hkv, L, D = 2, 8, 2, 1024, 128
    q = seeded((B, H, L, D), "bf16", 0.5)
    k = seeded((B, Hkv, L, D), "bf16", 0.5)
    v = seeded((B, Hkv, L, D), "bf16", 0.5)
    g = to_dev(seeded((B, H, L, D), "bf16"), "bf16")
    grads = []
    for _ in range(2):
        tq, tk, tv = (to_dev(x, "bf16", True) for x in (q, k, v))
        gtb.scaled_dot_product_attention(tq, tk, tv, is_causal=True).backward(g)
        grads.append((tq.grad.float(), tk.grad, tv.grad))
    (q1, k1, v1), (q2, k2, v2) = grads
    assert torch.equal(k1, k2) and torch.equal(v1, v2)
    assert torch.allclose(q1, q2, atol=1e-3, rtol=1e-2)


@pytest.mark.parametrize("dtype,B,H,Hkv,L,S,D,causal,chunk", [
    ("bf16", 5, 4, 2, 300, 300, 128, True, 2),    # three chunks, the last one ragged; tcgen05 path
    ("f32", 3, 2, 1, 70, 90, 64, False, None),    # default chunking (one sequence per chunk); SIMT path
    ("bf16", 2, 12, 3, 260, 260, 128, True, None),  # default chunking over kv heads (3 per sequence)
    ("bf16", 3, 10, 5, 129, 129, 128, False, None), # kv heads in ragged groups (3, 2 per sequence)
])
def test_sdpa_from_host_matches_the_device_call(dtype, B, H, Hkv, L, S, D, causal, chunk):
    """sdpa_from_host (pinned host tensors in and out, batch chunks pipelined over three streams)
    gives bit for bit what scaled_dot_product_attention gives on the same inputs in device memory."""
    import torch

    import gguf_train_b200 as gtb

    O.manual_seed(515 + B + L)
    q = to_dev(seeded((B, H, L, D), dtype, 0.5), dtype)
    k = to_dev(seeded((B, Hkv, S, D), dtype, 0.5), dtype)
    v = to_dev(seeded((B, Hkv, S, D), dtype, 0.5), dtype)
    want = gtb.scaled_dot_product_attention(q, k, v, is_causal=causal)
    qh, kh, vh = (x.cpu().pin_memory() for x in (q, k, v))
    got = gtb.sdpa_from_host(qh, kh, vh, is_causal=causal, chunk=chunk)
    torch.cuda.current_stream().synchronize()
    assert got.device.type == "cpu" and got.is_pinned()
    assert torch.equal(got, want.cpu())


def test_path_reports_the_kernel_family():
    """gtb_last_path names the kernels a call took: tcgen05 for 16-bit head size 128, the
    register-blocked fp32 kernels for fp32 head size 64, the one-warp-per-row kernels otherwise."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    for dtype, D, want in ((torch.bfloat16, 128, "tcgen05"), (torch.float32, 64, "f32_tiled"),
                           (torch.float32, 32, "simt")):
        q, k, v = (torch.randn(1, 2, 70, D, device="cuda", dtype=dtype, requires_grad=True) for _ in range(3))
        out = gtb.scaled_dot_product_attention(q, k, v, is_causal=True)
        assert _C.last_path() == want, (dtype, D, _C.last_path())
        out.sum().backward()
        assert _C.last_path() == want, (dtype, D, "backward", _C.last_path())
    assert _C.device_status() == 0
