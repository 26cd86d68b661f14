"""GPU parity of the Q8_0 codec (bit-exact) and of the Q8_0-cache decode step against the oracle."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import assert_close, seeded, to_dev

pytestmark = pytest.mark.gpu


def test_quantize_is_bit_exact_with_ggml():
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    O.manual_seed(3)
    x = (O.randn(64, 256) * 3.0).astype(np.float32)
    x[0, :32] = 0.0                       # an all-zero block: d = 0, id = 0
    x[1, :32] = np.linspace(-1, 1, 32)    # exact halves after scaling
    x[2, 5] = 1e-30                       # subnormal-range scale
    x[3, :32] = 65504.0 * 127             # scale above the fp16 range -> inf
    want = O.q8_0_quantize(x)
    got = gtb.quantize_q8_0(torch.tensor(x).cuda())
    assert _C.device_status() == 0
    assert np.array_equal(got.cpu().numpy().reshape(-1), want)
    # bf16 / f16 inputs quantise their (exactly representable) values the same way
    xb = O.round_to(x.astype(np.float64), O.BF16).astype(np.float32)
    gotb = gtb.quantize_q8_0(torch.tensor(xb).cuda().to(torch.bfloat16))
    assert np.array_equal(gotb.cpu().numpy().reshape(-1), O.q8_0_quantize(xb))


def test_dequantize_round_trip():
    import torch

    import gguf_train_b200 as gtb

    O.manual_seed(4)
    x = O.randn(8, 128).astype(np.float32)
    blocks = O.q8_0_quantize(x)
    dev = torch.tensor(blocks.reshape(8, 136)).cuda()
    got = gtb.dequantize_q8_0(dev, torch.float32).cpu().numpy()
    assert np.array_equal(got, O.q8_0_dequantize(blocks, (8, 128)))
    cos = float((got * x).sum() / np.sqrt((got * got).sum() * (x * x).sum()))
    assert cos > 0.999  # the reference's own check is cosine > 0.85 (test_gguf_and_llama.py:66-79)


def _decode_case(B, H, Hkv, Smax, D, lens, qdtype="f16", seed=5, kscale=1.0, vscale=1.0):
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    O.manual_seed(seed)
    q = seeded((B, H, 1, D), qdtype)
    kf = (O.randn(B, Hkv, Smax, D) * kscale).astype(np.float32)
    vf = (O.randn(B, Hkv, Smax, D) * vscale).astype(np.float32)
    kq = O.q8_0_quantize(kf)
    vq = O.q8_0_quantize(vf)
    want = O.decode_q8_0(q, kq, vq, np.asarray(lens, np.int32), Hkv, Smax)
    row = D // 32 * 34
    tk = torch.tensor(kq.reshape(B, Hkv, Smax, row)).cuda()
    tv = torch.tensor(vq.reshape(B, Hkv, Smax, row)).cuda()
    got = gtb.decode_q8_0(to_dev(q, qdtype), tk, tv, torch.tensor(lens, dtype=torch.int32).cuda())
    assert _C.device_status() == 0
    # outputs are compared in units of the V scale, so that the absolute tolerance keeps its meaning
    assert_close(got.double() / vscale, want / vscale, 2e-2, 1e-2,
                 f"decode B={B} H={H} Hkv={Hkv} Smax={Smax} D={D} lens={lens}")
    return got


@pytest.mark.parametrize("B,H,Hkv,Smax,D,lens", [
    (3, 8, 2, 300, 128, [1, 150, 300]),        # one chunk per sequence
    (2, 32, 8, 2500, 128, [2500, 1029]),       # several chunks: split-KV + combine
    (2, 4, 4, 64, 64, [64, 33]),               # D = 64, group of 1
    (1, 6, 2, 100, 128, [77]),                 # group of 3
    (2, 8, 1, 200, 256, [200, 5]),             # D = 256, group of 8 (split in two)
    (2, 4, 2, 301, 128, [301, 300]),           # odd Smax: word-wise staging instead of bulk copies
])
def test_decode_matches_oracle(B, H, Hkv, Smax, D, lens):
    _decode_case(B, H, Hkv, Smax, D, lens)


# D = 128 with an f16 query, H/Hkv in {1, 2, 4, 8} and an even Smax run on the tensor-core kernels
# (persistent CTAs, 64- or 128-row tiles, split-KV chunks of GTB_DECODE_CHUNK = 2048 rows; the plan
# lists full chunks first, then each sequence's partial last chunk by decreasing size): tile and
# chunk edges, group sizes, and rows past the end of a sequence inside a tile.
@pytest.mark.parametrize("B,H,Hkv,Smax,D,lens", [
    (4, 8, 8, 2050, 128, [1, 127, 128, 129]),           # group of 1, ragged first tiles
    (4, 16, 2, 2050, 128, [1023, 1024, 1025, 2050]),    # group of 8, tile edges, one full chunk + 2 rows
    (5, 32, 8, 6144, 128, [2047, 2048, 2049, 6144, 0]),  # group of 4, chunk edges: only full, only partial, both, empty
    (3, 8, 4, 4100, 128, [4100, 4094, 2]),              # group of 2, two full chunks + a partial one
    (3, 32, 8, 4096, 128, [4096, 2049, 640]),           # the config-5a group (4), several chunks
    (2, 4, 2, 256, 128, [256, 255]),                    # one chunk: normalised directly
])
def test_decode_tensor_core_path(B, H, Hkv, Smax, D, lens):
    _decode_case(B, H, Hkv, Smax, D, lens)


def test_decode_many_sequences():
    # more sequences than the plan kernel's 1024 threads: each thread scans a segment of lengths
    rng = np.random.default_rng(11)
    lens = rng.integers(0, 9, size=1100).tolist()
    _decode_case(1100, 4, 2, 8, 128, lens)


def test_decode_cache_scales():
    # tiny V scales (block scales near the f16 subnormal range) and large K scales (a peaked softmax)
    _decode_case(2, 8, 2, 600, 128, [600, 311], vscale=1e-5, kscale=30.0)
    _decode_case(2, 8, 2, 600, 128, [599, 1], vscale=300.0)


def test_decode_bf16_and_f32_queries():
    _decode_case(2, 8, 2, 700, 128, [700, 513], qdtype="bf16")
    _decode_case(2, 8, 2, 700, 128, [1, 699], qdtype="f32")


def test_decode_empty_sequence_gives_zero():
    got = _decode_case(2, 4, 2, 1100, 128, [0, 1100])
    assert float(got[0].abs().max()) == 0.0


def test_append_writes_the_quantised_rows_at_each_length():
    """q8_0_append quantises new rows into each sequence's cache rows [len, len + n_new), bit for bit
    as quantize_q8_0 (and so as ggml), leaves every other row alone and advances the lengths; a
    decode step then reads the appended rows (checked against the oracle)."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    O.manual_seed(61)
    B, H, Hkv, Smax, D, n_new = 3, 8, 2, 300, 128, 7
    lens = [5, 0, 290]
    base = (O.randn(B, Hkv, Smax, D) * 0.7).astype(np.float32)
    new = (O.randn(B, Hkv, n_new, D) * 0.7).astype(np.float32)
    cache = gtb.quantize_q8_0(torch.tensor(base).cuda())
    pos = torch.tensor(lens, dtype=torch.int32, device="cuda")
    gtb.q8_0_append(cache, torch.tensor(new).cuda().to(torch.bfloat16), pos)
    assert _C.device_status() == 0
    full = base.copy()
    new_bf = torch.tensor(new).to(torch.bfloat16).float().numpy()
    for b in range(B):
        full[b, :, lens[b]:lens[b] + n_new] = new_bf[b]
    want = O.q8_0_quantize(full.reshape(-1, D)).reshape(B, Hkv, Smax, D // 32 * 34)
    assert np.array_equal(cache.cpu().numpy(), want)
    assert pos.cpu().tolist() == [n + n_new for n in lens]
    # a decode step over the appended cache, against the oracle's dequantise-then-attend
    vq = O.q8_0_quantize(full.reshape(-1, D))
    vcache = torch.tensor(vq.reshape(B, Hkv, Smax, D // 32 * 34)).cuda()
    q = seeded((B, H, 1, D), "f16")
    got = gtb.decode_q8_0(to_dev(q, "f16"), cache, vcache, pos)
    assert _C.device_status() == 0
    ref = O.decode_q8_0(q, want.reshape(-1), vq, np.asarray(lens, np.int32) + n_new, Hkv, Smax)
    assert_close(got.double(), ref, 2e-2, 1e-2, "decode after append")


def test_append_past_the_cache_end_is_skipped_and_reported():
    """Rows that would land at or past Smax are not written; the kernel records status 60 and the
    rows that fit are written."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    O.manual_seed(62)
    B, Hkv, Smax, D, n_new = 1, 2, 64, 64, 4
    base = (O.randn(B, Hkv, Smax, D)).astype(np.float32)
    new = (O.randn(B, Hkv, n_new, D)).astype(np.float32)
    cache = gtb.quantize_q8_0(torch.tensor(base).cuda())
    before = cache.cpu().numpy().copy()
    pos = torch.tensor([Smax - 2], dtype=torch.int32, device="cuda")
    gtb.q8_0_append(cache, torch.tensor(new).cuda(), pos, advance=False)
    assert _C.device_status() == 60
    assert _C.device_status() == 0  # read and cleared
    got = cache.cpu().numpy()
    want_rows = O.q8_0_quantize(new[:, :, :2].reshape(-1, D)).reshape(B, Hkv, 2, D // 32 * 34)
    assert np.array_equal(got[:, :, Smax - 2:], want_rows)
    assert np.array_equal(got[:, :, :Smax - 2], before[:, :, :Smax - 2])
    assert pos.cpu().tolist() == [Smax - 2]


@pytest.mark.parametrize("dtype,B,H,S,D,n_dims,mode,base,fscale", [
    ("f32", 2, 3, 40, 64, 64, 0, 10000.0, 1.0),
    ("f32", 1, 4, 33, 128, 128, 2, 500000.0, 1.0),   # NeoX, llama-3 base
    ("f32", 2, 2, 17, 96, 32, 0, 10000.0, 0.25),     # partial rotation, linear position scaling
    ("bf16", 2, 8, 64, 128, 128, 2, 10000.0, 1.0),
    ("bf16", 2, 3, 70, 128, 128, 0, 10000.0, 1.0),   # 16-bit rows: normal mode, S not a multiple of 16
    ("f16", 1, 4, 33, 128, 64, 2, 500000.0, 1.0),    # 16-bit rows: NeoX, partial rotation
    ("f16", 2, 2, 17, 64, 32, 0, 10000.0, 0.25),
])
def test_rope_matches_oracle(dtype, B, H, S, D, n_dims, mode, base, fscale):
    """rope (forward) and its backward through RoPEFn against the oracle's restatement of ggml's
    rope, at positions up to 5000 (f32: 2e-5 abs; the angles, a few thousand radians, agree to the
    float ulp and CUDA's sincosf is within 2 ulp of the correctly rounded value; bf16: 2e-2 / 1e-2)."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    O.manual_seed(71 + S)
    x = seeded((B, H, S, D), dtype)
    g = seeded((B, H, S, D), dtype)
    pos = (np.arange(S) * 97 + 3) % 5000
    tx = to_dev(x, dtype, True)
    y = gtb.rope(tx, torch.tensor(pos, dtype=torch.int32).cuda(), n_dims, mode, 0, base, fscale)
    y.backward(to_dev(g, dtype))
    assert _C.device_status() == 0
    want = O.rope(x, pos, n_dims, mode, base, fscale)
    gwant = O.rope(g, pos, n_dims, mode, base, fscale, backward=True)
    atol, rtol = (2e-5, 1e-5) if dtype == "f32" else (2e-2, 1e-2)
    assert_close(y, want, atol, rtol, "rope forward")
    assert_close(tx.grad, gwant, atol, rtol, "rope backward")


@pytest.mark.parametrize("dtype,mode,n_dims", [("bf16", 0, 128), ("bf16", 2, 128), ("f16", 2, 64), ("f16", 0, 96)])
def test_rope_16bit_rows_equal_the_f32_path_rounded(dtype, mode, n_dims):
    """16-bit rows take the table-based kernel (angles computed once per position, 16-byte accesses);
    f32 rows take the per-pair kernel. Both form the same f32 angles and products, so the 16-bit
    result is bit for bit the f32 result on the same values rounded to the 16-bit type."""
    import torch

    import gguf_train_b200 as gtb

    B, H, S, D = 2, 4, 300, 128
    dt = torch.bfloat16 if dtype == "bf16" else torch.float16
    x = torch.randn(B, H, S, D, device="cuda").to(dt)
    pos = torch.tensor((np.arange(S) * 131 + 7) % 8000, dtype=torch.int32, device="cuda")
    got = gtb.rope(x, pos, n_dims, mode, 0, 10000.0, 1.0)
    ref = gtb.rope(x.float(), pos, n_dims, mode, 0, 10000.0, 1.0).to(dt)
    assert torch.equal(got, ref)


def test_append_with_rope_equals_rope_then_quantise():
    """q8_0_append with rope rotates each new row for its cache position and quantises the f32 result:
    for f32 rows that is bit for bit rope() at those positions followed by quantize_q8_0."""
    import torch

    import gguf_train_b200 as gtb
    from gguf_train_b200 import _C

    O.manual_seed(73)
    B, Hkv, Smax, D, n_new = 3, 2, 96, 128, 5
    lens = [0, 17, 90]
    cfg = dict(n_dims=128, mode=2, freq_base=10000.0, freq_scale=1.0)
    new = torch.tensor(O.randn(B, Hkv, n_new, D).astype(np.float32)).cuda()
    cache = torch.zeros((B, Hkv, Smax, D // 32 * 34), dtype=torch.uint8, device="cuda")
    pos = torch.tensor(lens, dtype=torch.int32, device="cuda")
    gtb.q8_0_append(cache, new, pos, rope=cfg)
    assert _C.device_status() == 0
    for b in range(B):
        positions = torch.arange(lens[b], lens[b] + n_new, dtype=torch.int32, device="cuda")
        rotated = gtb.rope(new[b:b + 1], positions, cfg["n_dims"], cfg["mode"], 0, cfg["freq_base"], cfg["freq_scale"])
        want = gtb.quantize_q8_0(rotated)
        assert torch.equal(cache[b:b + 1, :, lens[b]:lens[b] + n_new], want)
    assert pos.cpu().tolist() == [n + n_new for n in lens]
