"""Shared helpers of the parity tests: seeded inputs from the oracle's generator, tolerance checks."""

from __future__ import annotations

import numpy as np

from oracle import oracle as O

DT = {"f32": O.F32, "f16": O.F16, "bf16": O.BF16, "f64": O.F64}


def torch_dtype(name: str):
    import torch

    return {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16, "f64": torch.float64}[name]


def seeded(shape, dtype: str = "f32", scale: float = 1.0) -> np.ndarray:
    """N(0,1) * scale from the reference's generator, rounded to `dtype` (values as float64)."""
    return O.round_to(O.randn(*shape) * scale, DT[dtype])


def to_dev(x: np.ndarray, dtype: str, requires_grad: bool = False):
    import torch

    t = torch.tensor(x, dtype=torch.float64).to("cuda", torch_dtype(dtype))
    return t.requires_grad_() if requires_grad else t


def assert_close(got, want: np.ndarray, atol: float, rtol: float, what: str = "") -> float:
    import torch

    if isinstance(got, torch.Tensor):
        got = got.detach().double().cpu().numpy()
    got = np.asarray(got, dtype=np.float64)
    assert got.shape == want.shape, f"{what}: shape {got.shape} != {want.shape}"
    err = np.abs(got - want)
    bad = err > atol + rtol * np.abs(want)
    if bad.any():
        idx = np.unravel_index(np.argmax(err), err.shape)
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {err.size} elements outside atol={atol} rtol={rtol}; "
            f"max err {err.max():.3e} at {idx} (got {got[idx]:.6g}, want {want[idx]:.6g})"
        )
    return float(err.max()) if err.size else 0.0
