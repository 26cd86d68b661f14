"""The CPU restatement of gt_flash_attention pinned to the reference's own code.

oracle/_ref/ holds the reference's gt_flash_attention (csrc/gt_ops_nn.cpp:2423-2525) compiled from
its source (oracle/build_ref.py). The restatement in oracle/sdpa_oracle.cpp must give the same
stored results: bit for bit for f32/f16/bf16 outputs, and within 2 ulp for f64 (both accumulate in
double; the restatement's summation order may differ by a rounding).

Two forms: against the committed fixture that the reference produced
(tests/golden/make_ref_golden.py), which runs anywhere, and live against oracle/_ref where that
library exists (built here from the reference source; it travels with the tree)."""

from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_flash_attention.npz")


def _cases():
    data = np.load(GOLDEN)
    names = sorted({k.split("/")[0] for k in data.files})
    return data, names


def _restated(data, name):
    dt, causal, mdt, scale = data[f"{name}/args"]
    dt, mdt = int(dt), int(mdt)
    m = data[f"{name}/mask"] if f"{name}/mask" in data.files else None
    out = O.sdpa_fwd(data[f"{name}/q"], data[f"{name}/k"], data[f"{name}/v"], m, mdt == O.BOOL, float(scale),
                     bool(causal))
    return O.round_to(out, dt), dt


def _same(got, want, dt, what):
    if dt == O.F64:
        ulp = np.spacing(np.abs(want).max() + 1e-300)
        assert np.max(np.abs(got - want)) <= 2 * max(ulp, np.spacing(1.0)), what
    else:
        assert np.array_equal(got, want), f"{what}: max diff {np.max(np.abs(got - want)):.3e}"


def test_restatement_matches_the_reference_fixture():
    data, names = _cases()
    assert len(names) >= 10
    for name in names:
        got, dt = _restated(data, name)
        _same(got, data[f"{name}/out"], dt, name)


def test_fixture_covers_the_reference_rules():
    """The fixture exercises every rule of the reference loop: causal, GQA, L != S, bool and float
    masks with size-1 broadcasting, -inf entries and a fully masked row (output 0)."""
    data, names = _cases()
    out = data["bf16_float_4d_rows_masked/out"]
    assert np.all(out[:, 0, 3, :] == 0.0)  # the fully masked row gives 0 (gt_ops_nn.cpp:2509)
    assert data["f32_bool_kpm/mask"].shape == (2, 1, 1, 36)
    assert data["f32_float_bcast/mask"].shape == (2, 1, 40, 1)
    assert data["bf16_l_gt_s/q"].shape[2] > data["bf16_l_gt_s/k"].shape[2]


ref = pytest.importorskip("oracle.ref")


@pytest.mark.skipif(not ref.available(), reason="oracle/_ref not built and the reference source is absent")
def test_restatement_matches_the_reference_live():
    O.manual_seed(99)
    for dt in (O.F32, O.F16, O.BF16, O.F64):
        for causal, (B, H, Hkv, L, S, D) in ((True, (2, 4, 2, 37, 29, 24)), (False, (1, 6, 3, 21, 64, 16))):
            q = O.round_to(O.randn(B, H, L, D), dt)
            k = O.round_to(O.randn(B, Hkv, S, D), dt)
            v = O.round_to(O.randn(B, Hkv, S, D), dt)
            want = ref.flash_attention(q, k, v, dt, None, O.F32, 0.0, causal)
            got = O.round_to(O.sdpa_fwd(q, k, v, None, False, 0.0, causal), dt)
            _same(got, want, dt, f"dtype {dt} causal {causal}")
    # masks: bool (L, S), float (B, H, L, S) with -inf entries
    q, k, v = (O.round_to(O.randn(2, 4, 30, 8), O.F32) for _ in range(3))
    mb = (O.rand(30, 30) > 0.4).astype(np.float64)
    _same(O.round_to(O.sdpa_fwd(q, k, v, mb, True), O.F32), ref.flash_attention(q, k, v, O.F32, mb, O.BOOL), O.F32,
          "bool mask")
    mf = O.randn(2, 4, 30, 30)
    mf[O.rand(2, 4, 30, 30) < 0.1] = -np.inf
    mf = O.round_to(mf, O.F32)  # the values the reference reads from its f32 mask
    _same(O.round_to(O.sdpa_fwd(q, k, v, mf, False), O.F32), ref.flash_attention(q, k, v, O.F32, mf, O.F32), O.F32,
          "float mask")


@pytest.mark.skipif(not ref.available(), reason="oracle/_ref not built and the reference source is absent")
def test_decode_restatement_matches_the_reference_on_dequantised_caches():
    """The decode oracle = Q8_0 dequantisation (pinned bit-exact to gguf-py elsewhere) followed by
    gt_flash_attention over each sequence's first seq_lens[b] rows: checked here against the
    reference's function on the dequantised f32 caches."""
    O.manual_seed(5)
    B, H, Hkv, Smax, D = 3, 8, 2, 70, 64
    kq = O.q8_0_quantize(O.randn(B, Hkv, Smax, D))
    vq = O.q8_0_quantize(O.randn(B, Hkv, Smax, D))
    kd = O.q8_0_dequantize(kq, (B, Hkv, Smax, D)).astype(np.float64)
    vd = O.q8_0_dequantize(vq, (B, Hkv, Smax, D)).astype(np.float64)
    q = O.round_to(O.randn(B, H, 1, D), O.F16)
    lens = np.array([70, 1, 33], dtype=np.int32)
    got = O.decode_q8_0(q, kq.reshape(B, Hkv, Smax, -1), vq.reshape(B, Hkv, Smax, -1), lens, Hkv, Smax)
    for b in range(B):
        n = int(lens[b])
        want = ref.flash_attention(q[b:b + 1], kd[b:b + 1, :, :n], vd[b:b + 1, :, :n], O.F64)
        assert np.max(np.abs(got[b:b + 1] - want)) < 1e-12
