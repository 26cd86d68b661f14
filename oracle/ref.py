"""numpy front end of oracle/_ref/ -- TEST INFRASTRUCTURE ONLY.

oracle/_ref/libgt_ref_attn.so is the reference's own gt_flash_attention (csrc/gt_ops_nn.cpp:2423-2525)
compiled from its source by oracle/build_ref.py. Tests use it to pin the CPU restatement in
oracle/sdpa_oracle.cpp, and tests/golden/make_ref_golden.py records its outputs as fixtures so the
pin also holds where the reference source is absent.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import build_ref as _build_ref
from . import oracle as O

_lib = None

_NP = {O.F32: np.float32, O.F64: np.float64, O.F16: np.uint16, O.BF16: np.uint16, O.BOOL: np.uint8}


def available() -> bool:
    return _build_ref.available()


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = _build_ref.build()
        if path is None:
            raise RuntimeError("oracle/_ref is not built and the reference source is absent")
        L = ctypes.CDLL(str(path))
        P, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.ref_flash_attention.argtypes = [P, P, P, i32, i64, i64, i64, i64, i64, i64, i64, P, i32, i32, P,
                                          ctypes.c_float, i32, P]
        L.ref_flash_attention.restype = i32
        L.ref_last_error.restype = ctypes.c_char_p
        _lib = L
    return _lib


def _store(x, dtype: int) -> np.ndarray:
    """x (float64 values) in the storage format of `dtype` (bits for f16/bf16)."""
    if dtype in (O.F16, O.BF16, O.BOOL):
        return np.ascontiguousarray(O.to_bits(x, dtype))
    return np.ascontiguousarray(np.asarray(x, dtype=_NP[dtype]))


def flash_attention(q, k, v, dtype: int, mask=None, mask_dtype: int = O.F32, scale: float = 0.0,
                    is_causal: bool = False) -> np.ndarray:
    """The reference's gt_flash_attention on q, k, v (float64 values stored as `dtype`) and an
    optional 2-D or 4-D mask (stored as `mask_dtype`: BOOL, or a float type). Returns the output's
    float64 values as the reference stored them in `dtype`."""
    q, k, v = (np.asarray(t, dtype=np.float64) for t in (q, k, v))
    B, H, L, D = q.shape
    _, Hkv, S, Dv = v.shape
    qs, ks, vs = _store(q, dtype), _store(k, dtype), _store(v, dtype)
    out = np.zeros((B, H, L, Dv), dtype=_NP[dtype])
    if mask is not None:
        m = _store(mask, mask_dtype)
        mshape = np.asarray(m.shape, dtype=np.int64)
        margs = (m.ctypes.data, int(mask_dtype), m.ndim, mshape.ctypes.data)
    else:
        margs = (None, 0, 0, None)
    rc = lib().ref_flash_attention(qs.ctypes.data, ks.ctypes.data, vs.ctypes.data, int(dtype), B, H, L, D, Hkv, S,
                                   Dv, *margs, float(scale), int(bool(is_causal)), out.ctypes.data)
    if rc != 0:
        raise RuntimeError(lib().ref_last_error().decode())
    return O.from_bits(out, dtype) if dtype in (O.F16, O.BF16) else out.astype(np.float64)
