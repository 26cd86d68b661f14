"""numpy front end of the CPU oracle -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import this module, as the
checker and as the timed CPU baseline. The product package (gguf_train_b200) never imports it.

Each function names the reference behaviour it restates; the arithmetic lives in
oracle/sdpa_oracle.cpp. The forward is pinned to the reference's own gt_flash_attention, compiled
from its source into oracle/_ref/ (oracle/build_ref.py, tests/test_oracle_ref.py); the backward
and Q8_0 parts are pinned to independent implementations (see the C++ file's header).
"""

from __future__ import annotations

import ctypes
import math

import numpy as np

from . import build as _build

F32, F16, BF16, F64, BOOL = 0, 1, 2, 3, 9
_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = _build.build()
        L = ctypes.CDLL(str(path))
        P = ctypes.c_void_p
        i64, i32, f32, f64 = ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_double
        L.orc_manual_seed.argtypes = [ctypes.c_uint64]
        L.orc_fill_normal.argtypes = [P, i64, f64, f64]
        L.orc_fill_uniform.argtypes = [P, i64, f64, f64]
        L.orc_fill_bernoulli.argtypes = [P, i64, f64]
        L.orc_round_to_dtype.argtypes = [P, i64, i32, P]
        L.orc_to_bits.argtypes = [P, i64, i32, P]
        L.orc_from_bits.argtypes = [P, i64, i32, P]
        L.orc_sdpa_fwd.argtypes = [P, P, P, i64, i64, i64, i64, i64, i64, i64, P, i32, P, i32, f32, i32, P, i32]
        L.orc_sdpa_fwd_reforder.argtypes = [P, P, P, i64, i64, i64, i64, i64, i64, i64, f32, i32, i64, P, i32]
        L.orc_sdpa_bwd.argtypes = [P, P, P, P, i64, i64, i64, i64, i64, i64, i64, P, i32, P, i32, f64, i32, P, P, P, i32]
        L.orc_q8_0_quantize.argtypes = [P, i64, P]
        L.orc_q8_0_dequantize.argtypes = [P, i64, P]
        L.orc_decode_q8_0.argtypes = [P, P, P, P, i64, i64, i64, i64, i64, f32, P, i32]
        L.orc_num_threads.restype = i32
        L.orc_engine_raw.argtypes = [ctypes.c_uint64, i64, P]
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def _c64(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float64)


# ------------------------------------------------------------------ seeded inputs

def manual_seed(seed: int) -> None:
    """torch.manual_seed -> gt_manual_seed (gguf_train/_creation.py:343-347, gt_core.cpp:136-141)."""
    lib().orc_manual_seed(int(seed))


def randn(*shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    """torch.randn -> gt_fill_normal (gt_core.cpp:1199-1215): float64 draws, row-major."""
    out = np.empty(shape, dtype=np.float64)
    lib().orc_fill_normal(_p(out), out.size, float(mean), float(std))
    return out


def engine_raw(seed: int, n: int) -> np.ndarray:
    """The first n raw outputs of std::mt19937_64 seeded with `seed` (the reference's engine)."""
    out = np.empty(n, dtype=np.uint64)
    lib().orc_engine_raw(int(seed), int(n), _p(out))
    return out


def rand(*shape, low: float = 0.0, high: float = 1.0) -> np.ndarray:
    out = np.empty(shape, dtype=np.float64)
    lib().orc_fill_uniform(_p(out), out.size, float(low), float(high))
    return out


def bernoulli(*shape, p: float) -> np.ndarray:
    out = np.empty(shape, dtype=np.float64)
    lib().orc_fill_bernoulli(_p(out), out.size, float(p))
    return out


# ------------------------------------------------------------------ dtype storage

def round_to(x, dtype: int) -> np.ndarray:
    """The float64 value of x after it is stored in `dtype` (through float: gt_internal.h:261-266)."""
    x = _c64(x)
    out = np.empty_like(x)
    lib().orc_round_to_dtype(_p(x), x.size, int(dtype), _p(out))
    return out


def to_bits(x, dtype: int) -> np.ndarray:
    x = _c64(x)
    npdt = {F32: np.float32, F64: np.float64, F16: np.uint16, BF16: np.uint16, BOOL: np.uint8}[dtype]
    out = np.empty(x.shape, dtype=npdt)
    if lib().orc_to_bits(_p(x), x.size, int(dtype), _p(out)) != 0:
        raise ValueError(dtype)
    return out


def from_bits(b: np.ndarray, dtype: int) -> np.ndarray:
    b = np.ascontiguousarray(b)
    out = np.empty(b.shape, dtype=np.float64)
    if lib().orc_from_bits(_p(b), b.size, int(dtype), _p(out)) != 0:
        raise ValueError(dtype)
    return out


# ------------------------------------------------------------------ attention

def _mask_args(mask, is_bool):
    if mask is None:
        return None, 0, None, 0
    m = _c64(mask)
    if m.ndim not in (2, 4):
        raise ValueError("oracle mask must be 2-D or 4-D")
    shape = np.asarray(m.shape, dtype=np.int64)
    return m, m.ndim, shape, int(bool(is_bool))


def sdpa_fwd(q, k, v, mask=None, mask_is_bool=False, scale: float = 0.0, is_causal: bool = False,
             nthreads: int = 0) -> np.ndarray:
    """gt_flash_attention (csrc/gt_ops_nn.cpp:2423-2525) in float64; returns the double result
    before it is stored into q's dtype (round with round_to)."""
    q, k, v = _c64(q), _c64(k), _c64(v)
    B, H, L, D = q.shape
    _, Hkv, S, Dv = v.shape
    out = np.zeros((B, H, L, Dv), dtype=np.float64)
    m, mnd, msh, mb = _mask_args(mask, mask_is_bool)
    rc = lib().orc_sdpa_fwd(_p(q), _p(k), _p(v), B, H, Hkv, L, S, D, Dv,
                            _p(m) if m is not None else None, mnd, _p(msh) if msh is not None else None, mb,
                            float(scale), int(bool(is_causal)), _p(out), int(nthreads))
    if rc != 0:
        raise ValueError("oracle sdpa_fwd: bad shapes")
    return out


def sdpa_fwd_reforder(q, k, v, scale: float = 0.0, is_causal: bool = False, nthreads: int = 0,
                      q_offset: int = 0, out: np.ndarray | None = None) -> np.ndarray:
    """The same forward with the reference's literal loop order (the timed CPU baseline).
    q holds query rows q_offset.. of the sequence (causal masking uses absolute rows)."""
    q, k, v = _c64(q), _c64(k), _c64(v)
    B, H, L, D = q.shape
    _, Hkv, S, Dv = v.shape
    if out is None:
        out = np.zeros((B, H, L, Dv), dtype=np.float64)
    lib().orc_sdpa_fwd_reforder(_p(q), _p(k), _p(v), B, H, Hkv, L, S, D, Dv, float(scale),
                                int(bool(is_causal)), int(q_offset), _p(out), int(nthreads))
    return out


def sdpa_bwd(q, k, v, dout, mask=None, mask_is_bool=False, scale: float | None = None,
             is_causal: bool = False, nthreads: int = 0):
    """FlashAttentionFn.backward (gguf_train/_functions.py:1934-1965) in float64: (dq, dk, dv)."""
    q, k, v, dout = _c64(q), _c64(k), _c64(v), _c64(dout)
    B, H, L, D = q.shape
    _, Hkv, S, Dv = v.shape
    if scale is None or scale <= 0:
        scale = 1.0 / math.sqrt(D)
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    m, mnd, msh, mb = _mask_args(mask, mask_is_bool)
    rc = lib().orc_sdpa_bwd(_p(q), _p(k), _p(v), _p(dout), B, H, Hkv, L, S, D, Dv,
                            _p(m) if m is not None else None, mnd, _p(msh) if msh is not None else None, mb,
                            float(scale), int(bool(is_causal)), _p(dq), _p(dk), _p(dv), int(nthreads))
    if rc != 0:
        raise ValueError("oracle sdpa_bwd: bad shapes")
    return dq, dk, dv


# ------------------------------------------------------------------ Q8_0

def rope(x, pos, n_dims: int, mode: int = 0, freq_base: float = 10000.0, freq_scale: float = 1.0,
         backward: bool = False) -> np.ndarray:
    """gt_rope / gt_rope_backward (reference csrc/gt_ops_nn.cpp:2359-2421): ggml_rope_ext with
    ext_factor 0 and attn_factor 1 on x (..., S, D), one position per sequence element. Restates
    ggml's CPU rope (llama.cpp b12283, not vendored: the rope cache loop and rope_yarn) in float32:
    theta starts at p and is multiplied by theta_scale = powf(freq_base, -2/n_dims) after each pair,
    rotated angle = freq_scale * theta, mode 0 pairs (2i, 2i+1), mode 2 (NeoX) pairs (i, i + n_dims/2),
    x0' = x0 cos - x1 sin, x1' = x0 sin + x1 cos (sin negated for the backward); later dims copied.
    powf, cosf and sinf are taken as glibc gives them, correctly rounded: evaluated in float64 and
    rounded once (numpy's float32 power and trigonometry can be an ulp or more away)."""
    x = np.asarray(x, np.float32)
    out = x.copy()
    f32 = np.float32
    theta_scale = f32(np.float64(f32(freq_base)) ** (np.float64(f32(-2.0) / f32(n_dims))))
    half = n_dims // 2
    for s in range(x.shape[-2]):
        theta = f32(pos[s])
        for i in range(half):
            t = f32(f32(freq_scale) * theta)
            c, sn = f32(np.cos(np.float64(t))), f32(np.sin(np.float64(t)))
            if backward:
                sn = -sn
            c0, c1 = (i, i + half) if mode == 2 else (2 * i, 2 * i + 1)
            x0, x1 = x[..., s, c0], x[..., s, c1]
            out[..., s, c0] = x0 * c - x1 * sn
            out[..., s, c1] = x0 * sn + x1 * c
            theta = f32(theta * theta_scale)
    return out


def q8_0_quantize(x) -> np.ndarray:
    """Q8_0 blocks (34 B per 32 values) of x, rows along the last dim (gt_core.cpp:792-840)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if x.size % 32:
        raise ValueError("Q8_0 needs a multiple of 32 values")
    out = np.empty(x.size // 32 * 34, dtype=np.uint8)
    lib().orc_q8_0_quantize(_p(x), x.size, _p(out))
    return out


def q8_0_dequantize(blocks: np.ndarray, shape) -> np.ndarray:
    blocks = np.ascontiguousarray(blocks, dtype=np.uint8)
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    lib().orc_q8_0_dequantize(_p(blocks), n, _p(out))
    return out.reshape(shape)


def decode_q8_0(q, k_q8, v_q8, seq_lens, Hkv: int, Smax: int, scale: float = 0.0, nthreads: int = 0):
    """Q8_0 KV-cache decode: dequantize K/V to float32, then gt_flash_attention over each
    sequence's first seq_lens[b] rows. q (B, H, 1, D) float64; returns (B, H, 1, D) float64."""
    q = _c64(q)
    B, H, Lq, D = q.shape
    assert Lq == 1
    k_q8 = np.ascontiguousarray(k_q8, dtype=np.uint8)
    v_q8 = np.ascontiguousarray(v_q8, dtype=np.uint8)
    sl = np.ascontiguousarray(seq_lens, dtype=np.int32)
    out = np.zeros((B, H, 1, D), dtype=np.float64)
    rc = lib().orc_decode_q8_0(_p(q), _p(k_q8), _p(v_q8), _p(sl), B, H, Hkv, Smax, D, float(scale), _p(out),
                               int(nthreads))
    if rc != 0:
        raise ValueError("oracle decode: bad shapes")
    return out


def num_threads() -> int:
    return lib().orc_num_threads()
