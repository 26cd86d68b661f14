"""Generates the golden fixtures in tests/golden/ from implementations independent of this repo.

    python tests/golden/make_golden.py

* q8_0_gguf_py.npz: GGUF Q8_0 blocks from gguf-py (`gguf.quants.quantize`, whose Q8_0 class states
  bit-exactness with ggml-quants.c, the code the reference reaches through ggml_quantize_chunk) for
  seeded float32 rows, including an all-zero block and exact-half values.
* sdpa_torch_f64.npz: float64 attention outputs and gradients from real torch (CPU,
  torch.nn.functional.scaled_dot_product_attention and autograd) for small cases with GQA, causal
  masking (top-left), L != S, bool and float masks. The reference's semantics coincide with
  torch's on every row that keeps at least one key.

Inputs are drawn from numpy's PCG64 with fixed seeds (the fixtures store them).
"""

from __future__ import annotations

import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def q8_fixture():
    import gguf
    from gguf.quants import quantize

    rng = np.random.default_rng(8)
    x = (rng.standard_normal((16, 128)) * 3.0).astype(np.float32)
    x[0, :32] = 0.0
    x[1, :32] = np.linspace(-1.0, 1.0, 32, dtype=np.float32)
    x[2, :32] = np.float32(127.0) * (np.arange(32, dtype=np.float32) - 15.5)
    blocks = quantize(x, gguf.GGMLQuantizationType.Q8_0).reshape(-1)
    np.savez_compressed(os.path.join(HERE, "q8_0_gguf_py.npz"), x=x, blocks=blocks)


CASES = [
    # name, B, H, Hkv, L, S, D, causal, mask kind
    ("gqa_causal", 1, 4, 2, 16, 16, 8, True, None),
    ("lt_s_noncausal", 2, 2, 1, 5, 9, 8, False, None),
    ("gt_s_causal", 1, 2, 2, 9, 5, 16, True, None),
    ("bool_mask", 2, 3, 3, 4, 5, 6, False, "bool"),
    ("float_mask", 1, 2, 1, 7, 7, 8, False, "float"),
]


def sdpa_fixture():
    import torch

    out = {}
    rng = np.random.default_rng(9)
    for name, B, H, Hkv, L, S, D, causal, mk in CASES:
        q = rng.standard_normal((B, H, L, D))
        k = rng.standard_normal((B, Hkv, S, D))
        v = rng.standard_normal((B, Hkv, S, D))
        g = rng.standard_normal((B, H, L, D))
        mask = None
        if mk == "bool":
            mask = rng.random((B, 1, L, S)) < 0.7
            mask[..., 0] = True
        elif mk == "float":
            mask = rng.standard_normal((1, 1, L, S)) * 0.5
            drop = rng.random((1, 1, L, S)) < 0.2
            drop[..., 0] = False
            mask[drop] = -np.inf
        tq, tk, tv = (torch.tensor(a, requires_grad=True) for a in (q, k, v))
        rep = H // Hkv
        tmask = None
        if mask is not None:
            tmask = torch.tensor(mask)
        if causal:
            cm = torch.ones(L, S, dtype=torch.bool).tril()
            tmask = cm if tmask is None else (tmask & cm if tmask.dtype == torch.bool else tmask.masked_fill(~cm, -float("inf")))
        o = torch.nn.functional.scaled_dot_product_attention(
            tq, tk.repeat_interleave(rep, 1), tv.repeat_interleave(rep, 1), attn_mask=tmask)
        o.backward(torch.tensor(g))
        for key, val in dict(q=q, k=k, v=v, g=g, out=o.detach().numpy(), dq=tq.grad.numpy(), dk=tk.grad.numpy(),
                             dv=tv.grad.numpy()).items():
            out[f"{name}.{key}"] = val
        if mask is not None:
            out[f"{name}.mask"] = mask
    np.savez_compressed(os.path.join(HERE, "sdpa_torch_f64.npz"), **out)


if __name__ == "__main__":
    q8_fixture()
    sdpa_fixture()
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))
