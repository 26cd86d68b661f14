"""Regenerates tests/golden/ref_flash_attention.npz: outputs of the reference's own gt_flash_attention
(csrc/gt_ops_nn.cpp:2423-2525, compiled from its source by oracle/build_ref.py into oracle/_ref/)
on seeded inputs, so that tests/test_oracle_ref.py can pin the CPU restatement where the reference
source is absent (the GPU box). Run from the repository root:

    python tests/golden/make_ref_golden.py

Each case stores its inputs (float64 values already representable in the case's dtype), the mask,
the call's arguments and the reference's output (float64 values of what it stored in the dtype)."""

from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402
from oracle import ref as R  # noqa: E402

OUT = os.path.join(ROOT, "tests", "golden", "ref_flash_attention.npz")

# name, dtype, (B, H, Hkv, L, S, D, Dv), causal, mask kind, mask dtype, scale
CASES = [
    ("f32_causal_gqa", O.F32, (2, 4, 2, 33, 47, 16, 16), True, None, None, 0.0),
    ("f32_full", O.F32, (1, 2, 2, 20, 20, 8, 12), False, None, None, 0.3),
    ("f64_causal", O.F64, (1, 2, 1, 24, 24, 8, 8), True, None, None, 0.0),
    ("f16_causal_gqa", O.F16, (2, 4, 1, 17, 30, 32, 32), True, None, None, 0.0),
    ("bf16_causal_gqa", O.BF16, (2, 8, 2, 40, 40, 64, 64), True, None, None, 0.0),
    ("bf16_l_gt_s", O.BF16, (1, 4, 2, 50, 20, 16, 16), True, None, None, 0.0),
    ("f32_bool_2d", O.F32, (2, 4, 2, 40, 40, 8, 8), False, "bool2d", O.BOOL, 0.0),
    ("f32_bool_kpm", O.F32, (2, 4, 2, 24, 36, 8, 8), False, "bool_kpm", O.BOOL, 0.0),
    ("f32_float_bcast", O.F32, (2, 4, 2, 40, 40, 8, 8), False, "float_b1l1", O.F32, 0.0),
    ("bf16_float_4d_rows_masked", O.BF16, (2, 4, 2, 40, 40, 16, 16), True, "float_1hls_inf", O.BF16, 0.0),
    ("f16_bool_4d_causal", O.F16, (2, 2, 2, 33, 33, 32, 32), True, "bool_bhls", O.BOOL, 0.0),
]


def make_mask(kind, B, H, L, S):
    if kind is None:
        return None
    if kind == "bool2d":
        return (O.rand(L, S) > 0.3).astype(np.float64)
    if kind == "bool_kpm":  # key padding: the last n_b keys of sequence b may not be attended
        m = np.ones((B, 1, 1, S))
        for b in range(B):
            m[b, 0, 0, S - 3 - 5 * b:] = 0.0
        return m
    if kind == "float_b1l1":
        return O.randn(B, 1, L, 1)
    if kind == "float_1hls_inf":  # -inf at ~20% of the positions, and one row masked entirely
        m = O.randn(1, H, L, S)
        m[O.rand(1, H, L, S) < 0.2] = -np.inf
        m[0, 0, 3, :] = -np.inf
        return m
    if kind == "bool_bhls":
        return (O.rand(B, H, L, S) > 0.25).astype(np.float64)
    raise ValueError(kind)


def main():
    O.manual_seed(2024)
    data = {}
    for name, dt, (B, H, Hkv, L, S, D, Dv), causal, mk, mdt, scale in CASES:
        q = O.round_to(O.randn(B, H, L, D), dt)
        k = O.round_to(O.randn(B, Hkv, S, D), dt)
        v = O.round_to(O.randn(B, Hkv, S, Dv), dt)
        m = make_mask(mk, B, H, L, S)
        if m is not None and mdt != O.BOOL:
            m = O.round_to(m, mdt)
        out = R.flash_attention(q, k, v, dt, m, mdt if mdt is not None else O.F32, scale, causal)
        data[f"{name}/q"], data[f"{name}/k"], data[f"{name}/v"] = q, k, v
        data[f"{name}/args"] = np.array([dt, int(causal), -1 if mdt is None else mdt, scale], dtype=np.float64)
        if m is not None:
            data[f"{name}/mask"] = m
        data[f"{name}/out"] = out
    np.savez_compressed(OUT, **data)
    print(f"wrote {OUT}: {len(CASES)} cases")


if __name__ == "__main__":
    main()
