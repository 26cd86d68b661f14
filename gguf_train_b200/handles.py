"""Owned gt_tensor handles of the reference-shaped ABI (include/gguf_train_attn.h), with numpy I/O.

This is the calling convention of the reference's own Tensor class (gguf_train/_tensor.py:765-868:
a Python object owning a native handle, freed on __del__; results wrapped through check_ptr), kept
to what the attention exports need. Used by the C-ABI tests and by callers without torch.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _C

_NP_CODE = {
    np.dtype(np.float32): _C.GT_F32,
    np.dtype(np.float64): _C.GT_F64,
    np.dtype(np.float16): _C.GT_F16,
    np.dtype(np.int32): _C.GT_I32,
    np.dtype(np.int64): _C.GT_I64,
    np.dtype(np.bool_): _C.GT_BOOL,
    np.dtype(np.uint8): _C.GT_U8,
}


def _i64(vals):
    n = len(vals)
    return (ctypes.c_int64 * max(n, 1))(*vals)


class Handle:
    """An owned gt_tensor *."""

    def __init__(self, ptr: int, ctx: str = ""):
        self.ptr = _C.check_ptr(ptr, ctx)

    def __del__(self):
        ptr = getattr(self, "ptr", None)
        if ptr:
            _C.lib.gt_tensor_free(ptr)
            self.ptr = None

    # ---- metadata
    @property
    def shape(self):
        n = _C.lib.gt_tensor_ndim(self.ptr)
        buf = (ctypes.c_int64 * max(n, 1))()
        _C.lib.gt_tensor_shape(self.ptr, buf)
        return tuple(buf[i] for i in range(n))

    @property
    def dtype(self) -> int:
        return _C.lib.gt_tensor_dtype(self.ptr)

    @property
    def device_type(self) -> int:
        return _C.lib.gt_tensor_device_type(self.ptr)

    @property
    def nbytes(self) -> int:
        return _C.lib.gt_tensor_nbytes(self.ptr)

    # ---- construction
    @classmethod
    def empty(cls, shape, dtype: int, device: int = _C.GT_DEV_CUDA, index: int = 0) -> "Handle":
        return cls(_C.lib.gt_tensor_empty(len(shape), _i64(shape), dtype, device, index), "empty")

    @classmethod
    def from_numpy(cls, arr: np.ndarray, dtype: int | None = None, device: int = _C.GT_DEV_CUDA, index: int = 0,
                   shape=None) -> "Handle":
        """arr holds the raw element bytes (for bf16: uint16 bit patterns with dtype=GT_BF16;
        for Q8_0: uint8 blocks with dtype=GT_Q8_0 and the logical `shape`)."""
        arr = np.ascontiguousarray(arr)
        code = dtype if dtype is not None else _NP_CODE[arr.dtype]
        shp = tuple(arr.shape) if shape is None else tuple(shape)
        return cls(_C.lib.gt_tensor_from_data(len(shp), _i64(shp), code, device, index, arr.ctypes.data, arr.nbytes),
                   "from_data")

    def view(self, shape, strides, offset: int = 0) -> "Handle":
        return Handle(_C.lib.gt_tensor_view(self.ptr, len(shape), _i64(shape), _i64(strides), offset), "view")

    def to_numpy(self, np_dtype=None) -> np.ndarray:
        code = self.dtype
        if np_dtype is None:
            np_dtype = {_C.GT_F32: np.float32, _C.GT_F64: np.float64, _C.GT_F16: np.float16, _C.GT_BF16: np.uint16,
                        _C.GT_I32: np.int32, _C.GT_I64: np.int64, _C.GT_BOOL: np.bool_, _C.GT_U8: np.uint8,
                        _C.GT_Q8_0: np.uint8}[code]
        nb = self.nbytes
        out = np.empty(nb // np.dtype(np_dtype).itemsize, dtype=np_dtype)
        _C.check_rc(_C.lib.gt_tensor_copy_to_host(self.ptr, out.ctypes.data, nb), "copy_to_host")
        if code == _C.GT_Q8_0:
            return out
        return out.reshape(self.shape)


def flash_attention(q: Handle, k: Handle, v: Handle, mask: Handle | None = None, scale: float = 0.0,
                    is_causal: bool = False) -> Handle:
    return Handle(_C.lib.gt_flash_attention(q.ptr, k.ptr, v.ptr, mask.ptr if mask else None, scale, int(is_causal)),
                  "flash_attention")


def flash_attention_fwd_lse(q, k, v, mask=None, scale: float = 0.0, is_causal: bool = False):
    lse = ctypes.c_void_p()
    out = Handle(_C.lib.gt_flash_attention_fwd_lse(q.ptr, k.ptr, v.ptr, mask.ptr if mask else None, scale,
                                                   int(is_causal), ctypes.byref(lse)), "flash_attention")
    return out, Handle(lse.value, "flash_attention")


def flash_attention_backward(grad_out, q, k, v, mask, out, lse, scale: float = 0.0, is_causal: bool = False):
    dq, dk, dv = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
    rc = _C.lib.gt_flash_attention_backward(grad_out.ptr, q.ptr, k.ptr, v.ptr, mask.ptr if mask else None, out.ptr,
                                            lse.ptr, scale, int(is_causal), ctypes.byref(dq), ctypes.byref(dk),
                                            ctypes.byref(dv))
    _C.check_rc(rc, "flash_attention_backward")
    return Handle(dq.value), Handle(dk.value), Handle(dv.value)


def rope(x: Handle, pos: Handle, n_dims: int, mode: int = 0, n_ctx_orig: int = 0, freq_base: float = 10000.0,
         freq_scale: float = 1.0, backward: bool = False) -> Handle:
    fn = _C.lib.gt_rope_backward if backward else _C.lib.gt_rope
    return Handle(fn(x.ptr, pos.ptr, n_dims, mode, n_ctx_orig, freq_base, freq_scale), "rope")


def quantize(t: Handle, qtype: int = _C.GT_Q8_0) -> Handle:
    return Handle(_C.lib.gt_quantize(t.ptr, qtype), "quantize")


def dequantize(t: Handle, dtype: int = _C.GT_F32) -> Handle:
    return Handle(_C.lib.gt_dequantize(t.ptr, dtype), "dequantize")


def flash_decode_q8_0(q: Handle, k_q8: Handle, v_q8: Handle, seq_lens: Handle, scale: float = 0.0) -> Handle:
    return Handle(_C.lib.gt_flash_decode_q8_0(q.ptr, k_q8.ptr, v_q8.ptr, seq_lens.ptr, scale), "flash_decode_q8_0")
