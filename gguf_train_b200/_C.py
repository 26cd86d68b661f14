"""ctypes binding of the engine's C ABI (include/gtb_attn.h and include/gguf_train_attn.h).

Mirrors the reference's loader, gguf_train/_C.py: the library is opened with ctypes.CDLL
(:204-206), every export gets argtypes/restype (the attention binding is the reference's own,
:471-472: [c_void_p x4, c_float, c_int] -> c_void_p), and a NULL pointer or non-zero return code is
raised as an exception carrying the thread-local native message (check_ptr / check_rc,
:688-710; an "IndexError: " prefix becomes IndexError).

There is no fallback: if the library is missing or cannot be loaded, importing this module raises.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

_PKG = Path(__file__).resolve().parent
_LIB_PATH = _PKG / "_lib" / "libgt_attn_b200.so"

c_void_p = ctypes.c_void_p
c_int = ctypes.c_int
c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64
c_uint64 = ctypes.c_uint64
c_size_t = ctypes.c_size_t
c_float = ctypes.c_float
c_double = ctypes.c_double
c_char_p = ctypes.c_char_p
p_i64 = ctypes.POINTER(c_int64)

# gt_dtype codes (reference csrc/gguf_train.h:22-36, gguf_train/_dtype.py:85)
GT_F32, GT_F16, GT_BF16, GT_F64, GT_I8, GT_U8, GT_I16, GT_I32, GT_I64, GT_BOOL = 0, 1, 2, 3, 4, 5, 6, 7, 8, 9
GTB_BWD_DETERMINISTIC = 1  # gtb_sdpa_bwd_ex flag (include/gtb_attn.h)
GT_Q8_0 = 108
GT_DEV_CPU, GT_DEV_CUDA = 0, 1


class Tensor4(ctypes.Structure):
    """gtb_tensor4: a strided 4-D view of device memory (include/gtb_attn.h)."""

    _fields_ = [("data", c_void_p), ("shape", c_int64 * 4), ("stride", c_int64 * 4), ("dtype", c_int32)]


P4 = ctypes.POINTER(Tensor4)


class SdpaOpts(ctypes.Structure):
    """gtb_sdpa_opts (include/gtb_attn.h): flags, dropout probability, dropout seed."""
    _fields_ = [("flags", ctypes.c_int32), ("dropout_p", ctypes.c_float), ("dropout_seed", ctypes.c_uint64)]


POPTS = ctypes.POINTER(SdpaOpts)


def _configure(lib: ctypes.CDLL) -> ctypes.CDLL:
    # raw-pointer ABI (gtb_attn.h)
    lib.gtb_sdpa_fwd.argtypes = [P4, P4, P4, P4, c_float, c_int, P4, c_void_p, c_void_p]
    lib.gtb_sdpa_fwd_ex.argtypes = [P4, P4, P4, P4, c_float, c_int, P4, c_void_p, POPTS, c_void_p]
    lib.gtb_sdpa_fwd_ex.restype = c_int
    lib.gtb_sdpa_fwd_rope.argtypes = [P4, P4, P4, P4, c_float, c_int, c_void_p, c_int64, c_void_p, c_int64, c_int, c_int,
                                      c_float, c_float, c_int, P4, P4, c_void_p, c_void_p]
    lib.gtb_sdpa_fwd_rope.restype = c_int
    lib.gtb_attn_weights.argtypes = [P4, P4, P4, c_void_p, c_float, c_int, c_int, POPTS, P4, c_void_p]
    lib.gtb_attn_weights.restype = c_int
    lib.gtb_linear.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64, c_int64, c_int64,
                               c_int64, c_int, c_void_p]
    lib.gtb_linear.restype = c_int
    lib.gtb_sdpa_fwd.restype = c_int
    lib.gtb_sdpa_fwd_host.argtypes = [P4, P4, P4, c_float, c_int, P4, c_int, c_void_p]
    lib.gtb_sdpa_fwd_host.restype = c_int
    lib.gtb_sdpa_bwd.argtypes = [P4, P4, P4, P4, P4, P4, c_void_p, c_float, c_int, P4, P4, P4, c_void_p]
    lib.gtb_sdpa_bwd.restype = c_int
    lib.gtb_sdpa_bwd_ex.argtypes = [P4, P4, P4, P4, P4, P4, c_void_p, c_float, c_int, P4, P4, P4, POPTS, c_void_p]
    lib.gtb_sdpa_bwd_ex.restype = c_int
    lib.gtb_q8_0_quantize.argtypes = [c_void_p, c_int, c_int64, c_int64, c_void_p, c_void_p]
    lib.gtb_q8_0_quantize.restype = c_int
    lib.gtb_q8_0_append.argtypes = [c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, c_void_p, c_int64, c_void_p,
                                    c_int, c_void_p]
    lib.gtb_q8_0_append.restype = c_int
    lib.gtb_q8_0_append_rope.argtypes = [c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, c_void_p, c_int64,
                                         c_void_p, c_int, c_int, c_int, c_float, c_float, c_void_p]
    lib.gtb_q8_0_append_rope.restype = c_int
    lib.gtb_rope.argtypes = [c_void_p, c_int, c_int64, c_int64, c_int64, c_int64, c_void_p, c_int64, c_int, c_int,
                             c_float, c_float, c_int, c_void_p, c_void_p]
    lib.gtb_rope.restype = c_int
    lib.gtb_q8_0_dequantize.argtypes = [c_void_p, c_int64, c_int64, c_void_p, c_int, c_void_p]
    lib.gtb_q8_0_dequantize.restype = c_int
    lib.gtb_decode_q8_0.argtypes = [c_void_p, c_int, c_void_p, c_void_p, c_void_p, c_int64, c_int64, c_int64,
                                    c_int64, c_int64, c_float, c_void_p, c_void_p]
    lib.gtb_decode_q8_0.restype = c_int
    lib.gtb_decode_q8_0_noalloc.argtypes = list(lib.gtb_decode_q8_0.argtypes)
    lib.gtb_decode_q8_0_noalloc.restype = c_int
    lib.gtb_attn_merge.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int64, c_int64, c_int64, c_int64,
                                   c_int64, c_void_p]
    lib.gtb_attn_merge.restype = c_int
    lib.gtb_last_error.argtypes = []
    lib.gtb_last_error.restype = c_char_p
    lib.gtb_clear_error.argtypes = []
    lib.gtb_clear_error.restype = None
    lib.gtb_device_status.argtypes = []
    lib.gtb_device_status.restype = c_int
    lib.gtb_selftest_wait_timeout.argtypes = [c_int64, c_void_p]
    lib.gtb_selftest_wait_timeout.restype = c_int
    lib.gtb_version.argtypes = []
    lib.gtb_version.restype = c_char_p
    lib.gtb_last_path.argtypes = []
    lib.gtb_last_path.restype = c_char_p

    # handle ABI (gguf_train_attn.h), argtypes as the reference binds them
    lib.gt_last_error.argtypes = []
    lib.gt_last_error.restype = c_char_p
    lib.gt_clear_error.argtypes = []
    lib.gt_clear_error.restype = None
    lib.gt_manual_seed.argtypes = [c_uint64]
    lib.gt_manual_seed.restype = None
    lib.gt_device_count.argtypes = [c_int]
    lib.gt_device_count.restype = c_int
    lib.gt_device_name.argtypes = [c_int, c_int, c_char_p, c_int]
    lib.gt_device_name.restype = None
    lib.gt_device_memory.argtypes = [c_int, c_int, ctypes.POINTER(c_size_t), ctypes.POINTER(c_size_t)]
    lib.gt_device_memory.restype = None
    lib.gt_synchronize.argtypes = [c_int, c_int]
    lib.gt_synchronize.restype = None
    lib.gt_tensor_empty.argtypes = [c_int, p_i64, c_int, c_int, c_int]
    lib.gt_tensor_empty.restype = c_void_p
    lib.gt_tensor_from_data.argtypes = [c_int, p_i64, c_int, c_int, c_int, c_void_p, c_size_t]
    lib.gt_tensor_from_data.restype = c_void_p
    lib.gt_tensor_from_external.argtypes = [c_int, p_i64, p_i64, c_int, c_void_p, c_uint64]
    lib.gt_tensor_from_external.restype = c_void_p
    lib.gt_tensor_clone.argtypes = [c_void_p]
    lib.gt_tensor_clone.restype = c_void_p
    lib.gt_tensor_view.argtypes = [c_void_p, c_int, p_i64, p_i64, c_int64]
    lib.gt_tensor_view.restype = c_void_p
    lib.gt_tensor_contiguous.argtypes = [c_void_p]
    lib.gt_tensor_contiguous.restype = c_void_p
    lib.gt_tensor_to_dtype.argtypes = [c_void_p, c_int]
    lib.gt_tensor_to_dtype.restype = c_void_p
    lib.gt_tensor_to_device.argtypes = [c_void_p, c_int, c_int]
    lib.gt_tensor_to_device.restype = c_void_p
    lib.gt_tensor_free.argtypes = [c_void_p]
    lib.gt_tensor_free.restype = None
    lib.gt_tensor_ndim.argtypes = [c_void_p]
    lib.gt_tensor_ndim.restype = c_int
    lib.gt_tensor_shape.argtypes = [c_void_p, p_i64]
    lib.gt_tensor_shape.restype = None
    lib.gt_tensor_strides.argtypes = [c_void_p, p_i64]
    lib.gt_tensor_strides.restype = None
    lib.gt_tensor_offset.argtypes = [c_void_p]
    lib.gt_tensor_offset.restype = c_int64
    lib.gt_tensor_numel.argtypes = [c_void_p]
    lib.gt_tensor_numel.restype = c_int64
    lib.gt_tensor_dtype.argtypes = [c_void_p]
    lib.gt_tensor_dtype.restype = c_int
    lib.gt_tensor_device_type.argtypes = [c_void_p]
    lib.gt_tensor_device_type.restype = c_int
    lib.gt_tensor_device_index.argtypes = [c_void_p]
    lib.gt_tensor_device_index.restype = c_int
    lib.gt_tensor_is_contiguous.argtypes = [c_void_p]
    lib.gt_tensor_is_contiguous.restype = c_int
    lib.gt_tensor_data_ptr.argtypes = [c_void_p]
    lib.gt_tensor_data_ptr.restype = c_uint64
    lib.gt_tensor_nbytes.argtypes = [c_void_p]
    lib.gt_tensor_nbytes.restype = c_size_t
    lib.gt_tensor_elem_size.argtypes = [c_int]
    lib.gt_tensor_elem_size.restype = c_size_t
    lib.gt_tensor_copy_to_host.argtypes = [c_void_p, c_void_p, c_size_t]
    lib.gt_tensor_copy_to_host.restype = c_int
    lib.gt_tensor_copy_from_host.argtypes = [c_void_p, c_void_p, c_size_t]
    lib.gt_tensor_copy_from_host.restype = c_int
    lib.gt_fill_uniform.argtypes = [c_void_p, c_double, c_double]
    lib.gt_fill_uniform.restype = c_int
    lib.gt_fill_normal.argtypes = [c_void_p, c_double, c_double]
    lib.gt_fill_normal.restype = c_int
    lib.gt_fill_bernoulli_prob.argtypes = [c_void_p, c_double]
    lib.gt_fill_bernoulli_prob.restype = c_int
    lib.gt_flash_attention.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_int]
    lib.gt_flash_attention.restype = c_void_p
    lib.gt_flash_attention_fwd_lse.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_float, c_int,
                                               ctypes.POINTER(c_void_p)]
    lib.gt_flash_attention_fwd_lse.restype = c_void_p
    lib.gt_flash_attention_backward.argtypes = [c_void_p] * 7 + [c_float, c_int] + [ctypes.POINTER(c_void_p)] * 3
    lib.gt_flash_attention_backward.restype = c_int
    lib.gt_flash_decode_q8_0.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_float]
    lib.gt_flash_decode_q8_0.restype = c_void_p
    lib.gt_rope.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float]
    lib.gt_rope.restype = c_void_p
    lib.gt_rope_backward.argtypes = [c_void_p, c_void_p, c_int, c_int, c_int, c_float, c_float]
    lib.gt_rope_backward.restype = c_void_p
    lib.gt_quantize.argtypes = [c_void_p, c_int]
    lib.gt_quantize.restype = c_void_p
    lib.gt_dequantize.argtypes = [c_void_p, c_int]
    lib.gt_dequantize.restype = c_void_p
    return lib


def _load() -> ctypes.CDLL:
    path = Path(os.environ.get("GTB_LIB", str(_LIB_PATH)))
    if not path.exists():
        raise ImportError(
            f"gguf_train_b200: native library {path} is missing; build it with "
            "`python -c 'import __graft_entry__ as g; g.build()'` (nvcc, sm_100a)"
        )
    return _configure(ctypes.CDLL(str(path)))


lib = _load()
LIB_PATH = str(_LIB_PATH)


def last_error() -> str:
    msg = lib.gt_last_error()
    return msg.decode("utf-8", errors="replace") if msg else ""


_NATIVE_ERROR_TYPES = {"IndexError": IndexError}


def _native_error(ctx: str, err: str, fallback: str) -> Exception:
    for name, exc_type in _NATIVE_ERROR_TYPES.items():
        tag = name + ": "
        if err.startswith(tag):
            return exc_type(err[len(tag):])
    if ctx and err:
        return RuntimeError(err if err.startswith(ctx + ":") or err.startswith(ctx + " ") else f"{ctx}: {err}")
    return RuntimeError(err or ctx or fallback)


def check_ptr(ptr, ctx: str = "") -> int:
    if not ptr:
        raise _native_error(ctx, last_error(), "Native operation returned NULL")
    return ptr


def check_rc(rc: int, ctx: str = "") -> None:
    if rc != 0:
        raise _native_error(ctx, last_error(), f"Native operation failed with code {rc}")


def device_status() -> int:
    """Synchronise and read (then clear) the device's kernel status word (0 = no timeout)."""
    return lib.gtb_device_status()


def last_path() -> str:
    """Kernel family ("tcgen05" or "simt") of this thread's last native attention forward/backward."""
    return lib.gtb_last_path().decode()
