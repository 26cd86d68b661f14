"""The native library without a GPU: it loads, exports every symbol its headers declare, keeps the
reference's handle and error conventions, and refuses CPU tensors on the attention path."""

from __future__ import annotations

import ctypes
import os
import re

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header: str, macro: str):
    text = open(os.path.join(ROOT, "include", header)).read()
    text = "\n".join(line for line in text.splitlines() if not line.lstrip().startswith("#"))
    return sorted(set(re.findall(macro + r"\s+[^;(]*?\b(\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    from gguf_train_b200 import _C

    names = _declared("gtb_attn.h", "GTB_API") + _declared("gguf_train_attn.h", "GT_API")
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(_C.lib, n)]
    assert not missing, missing


def test_library_is_built_for_sm_100a_only():
    from gguf_train_b200 import _C

    assert b"sm_100a" in _C.lib.gtb_version()
    # the build passes exactly one -gencode, for sm_100a
    from gguf_train_b200 import _build

    assert _build.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]


def test_handles_round_trip_views_and_contiguous():
    from gguf_train_b200 import _C
    from gguf_train_b200.handles import Handle

    a = np.arange(24, dtype=np.float32).reshape(2, 3, 4)
    h = Handle.from_numpy(a, device=_C.GT_DEV_CPU)
    assert h.shape == (2, 3, 4) and h.dtype == _C.GT_F32 and h.device_type == _C.GT_DEV_CPU
    assert np.array_equal(h.to_numpy(), a)
    t = h.view((4, 3, 2), (1, 4, 12))                      # the full transpose as a view
    assert np.array_equal(t.to_numpy(), a.transpose(2, 1, 0))
    c = Handle(_C.lib.gt_tensor_contiguous(t.ptr))
    assert _C.lib.gt_tensor_is_contiguous(c.ptr) == 1
    assert np.array_equal(c.to_numpy(), a.transpose(2, 1, 0))
    off = h.view((3, 4), (4, 1), 12)                       # a[1] through an element offset
    assert np.array_equal(off.to_numpy(), a[1])


def test_seeded_fill_matches_the_reference_generator():
    """gt_manual_seed + gt_fill_normal (gt_core.cpp:136-141, 1199-1215): the same libstdc++
    mt19937_64 / normal_distribution<double> draws as the oracle's restatement, stored through float."""
    from gguf_train_b200 import _C
    from gguf_train_b200.handles import Handle
    from oracle import oracle as O

    h = Handle.empty((3, 5, 7), _C.GT_F32, _C.GT_DEV_CPU)
    _C.lib.gt_manual_seed(0)
    _C.check_rc(_C.lib.gt_fill_normal(h.ptr, 0.0, 1.0), "fill_normal")
    O.manual_seed(0)
    assert np.array_equal(h.to_numpy(), O.randn(3, 5, 7).astype(np.float32))
    hb = Handle.empty((64,), _C.GT_BF16, _C.GT_DEV_CPU)
    _C.lib.gt_manual_seed(3)
    _C.lib.gt_fill_normal(hb.ptr, 0.0, 0.5)
    O.manual_seed(3)
    assert np.array_equal(hb.to_numpy(), O.to_bits(O.randn(64) * 0.5, O.BF16))


def test_attention_refuses_cpu_tensors_with_the_reference_error_style():
    from gguf_train_b200 import _C
    from gguf_train_b200 import handles as H

    q = H.Handle.from_numpy(np.zeros((1, 2, 4, 8), np.float32), device=_C.GT_DEV_CPU)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        H.flash_attention(q, q, q)
    bad = H.Handle.from_numpy(np.zeros((2, 4, 8), np.float32), device=_C.GT_DEV_CPU)
    with pytest.raises(RuntimeError, match=r"flash_attention expects 4D q, k, v tensors \(B, H, L, D\)"):
        H.flash_attention(bad, bad, bad)
    # a NULL result leaves the message in the thread-local slot until cleared (gt_core.cpp:7-23)
    assert "4D" in _C.last_error()
    _C.lib.gt_clear_error()
    assert _C.last_error() == ""


def test_raw_abi_rejects_host_pointers_and_bad_shapes():
    from gguf_train_b200 import _C

    host = np.zeros((1, 2, 4, 8), np.float32)

    def t4(arr, shape=None):
        t = _C.Tensor4()
        t.data = arr.ctypes.data
        for i, (s, st) in enumerate(zip(shape or arr.shape, np.array(arr.strides) // arr.itemsize)):
            t.shape[i], t.stride[i] = s, int(st)
        t.dtype = _C.GT_F32
        return t

    q, out = t4(host), t4(host.copy())
    rc = _C.lib.gtb_sdpa_fwd(ctypes.byref(q), ctypes.byref(q), ctypes.byref(q), None, 0.0, 0, ctypes.byref(out),
                             None, None)
    assert rc != 0 and "no CPU path" in _C.lib.gtb_last_error().decode()
    k3 = t4(np.zeros((1, 3, 4, 8), np.float32))
    rc = _C.lib.gtb_sdpa_fwd(ctypes.byref(q), ctypes.byref(k3), ctypes.byref(k3), None, 0.0, 0, ctypes.byref(out),
                             None, None)
    assert rc != 0 and "num_heads must be divisible by num_kv_heads" in _C.lib.gtb_last_error().decode()
    m = t4(np.zeros((1, 1, 3, 4), np.float32))
    rc = _C.lib.gtb_sdpa_fwd(ctypes.byref(q), ctypes.byref(q), ctypes.byref(q), ctypes.byref(m), 0.0, 0,
                             ctypes.byref(out), None, None)
    assert rc != 0 and "cannot be broadcast" in _C.lib.gtb_last_error().decode()
    rc = _C.lib.gtb_q8_0_quantize(host.ctypes.data, _C.GT_F32, 1, 33, host.ctypes.data, None)
    assert rc != 0 and "multiple of ggml quantization block size" in _C.lib.gtb_last_error().decode()


def test_host_forward_argument_checks():
    """gtb_sdpa_fwd_host (host q, k, v, out) checks shapes, dtypes and layout before any device work."""
    from gguf_train_b200 import _C

    def t4(arr, shape=None, strides=None):
        t = _C.Tensor4()
        t.data = arr.ctypes.data
        sts = strides or [int(s) for s in np.array(arr.strides) // arr.itemsize]
        for i, (s, st) in enumerate(zip(shape or arr.shape, sts)):
            t.shape[i], t.stride[i] = s, st
        t.dtype = _C.GT_F32
        return t

    q = np.zeros((1, 2, 4, 8), np.float32)
    k3 = np.zeros((1, 3, 4, 8), np.float32)

    def call(qq, kk, vv, oo):
        rc = _C.lib.gtb_sdpa_fwd_host(ctypes.byref(qq), ctypes.byref(kk), ctypes.byref(vv), 0.0, 0, ctypes.byref(oo),
                                      0, None)
        return rc, _C.lib.gtb_last_error().decode()

    rc, msg = call(t4(q), t4(k3), t4(k3), t4(q.copy()))
    assert rc != 0 and "num_heads must be divisible by num_kv_heads" in msg
    rc, msg = call(t4(q), t4(q), t4(q), t4(np.zeros((1, 2, 4, 4), np.float32)))
    assert rc != 0 and "out must be" in msg
    # a (B, H, L, D) view whose L and D strides are swapped is not row-major
    rc, msg = call(t4(q, (1, 2, 4, 8), [64, 32, 1, 4]), t4(q), t4(q), t4(q.copy()))
    assert rc != 0 and "contiguous (row-major)" in msg


def test_q8_0_append_argument_checks():
    """gtb_q8_0_append rejects a row length that is not whole Q8_0 blocks, negative sizes and
    non-float rows before any device work."""
    from gguf_train_b200 import _C

    def call(D=64, dtype=_C.GT_F32, n_new=1):
        rc = _C.lib.gtb_q8_0_append(None, dtype, 1, 1, n_new, D, None, 8, None, 1, None)
        return rc, _C.lib.gtb_last_error().decode()

    rc, msg = call(D=33)
    assert rc != 0 and "multiple of ggml quantization block size" in msg
    rc, msg = call(n_new=-1)
    assert rc != 0 and "negative size" in msg
    rc, msg = call(dtype=_C.GT_F64)
    assert rc != 0 and "f32, f16 or bf16" in msg
    assert call(n_new=0)[0] == 0  # nothing to append


def test_rope_argument_checks_use_the_reference_messages():
    """gtb_rope checks mode, n_dims, the frequencies and the positions with gt_rope_check's messages
    (csrc/gt_ops_nn.cpp:2316-2357) before any device work."""
    from gguf_train_b200 import _C

    def call(mode=0, n_dims=8, base=10000.0, n_pos=4):
        rc = _C.lib.gtb_rope(None, _C.GT_F32, 1, 1, 4, 8, None, n_pos, n_dims, mode, base, 1.0, 0, None, None)
        return rc, _C.lib.gtb_last_error().decode()

    rc, msg = call(mode=1)
    assert rc != 0 and "mode must be 0 (normal) or 2 (NeoX)" in msg
    rc, msg = call(n_dims=3)
    assert rc != 0 and "n_dims must be an even number between 2 and the head dimension 8" in msg
    rc, msg = call(n_dims=10)
    assert rc != 0 and "n_dims must be an even number" in msg
    rc, msg = call(base=0.0)
    assert rc != 0 and "freq_base must be positive and finite" in msg
    rc, msg = call(n_pos=3)
    assert rc != 0 and "a position for each of the 4 sequence elements" in msg


def test_handle_rope_checks():
    """gt_rope (the reference's own ctypes signature) reports a bad rank with gt_rope_check's message
    and refuses host tensors: the engine has no CPU path."""
    import gguf_train_b200.handles as H
    from gguf_train_b200 import _C

    pos = H.Handle.from_numpy(np.arange(4, dtype=np.int32), device=_C.GT_DEV_CPU)
    bad = H.Handle.from_numpy(np.zeros((4, 8), np.float32), device=_C.GT_DEV_CPU)
    with pytest.raises(RuntimeError, match=r"rope: expected x of shape .* got \[4, 8\]"):
        H.rope(bad, pos, 8)
    x = H.Handle.from_numpy(np.zeros((1, 2, 4, 8), np.float32), device=_C.GT_DEV_CPU)
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        H.rope(x, pos, 8)


def test_fused_rope_forward_argument_checks():
    """gtb_sdpa_fwd_rope checks the attention shapes, the rope arguments, the positions and k_rot
    before any device work."""
    from gguf_train_b200 import _C

    def t4(arr, dtype=None):
        t = _C.Tensor4()
        t.data = arr.ctypes.data
        for i, (s, st) in enumerate(zip(arr.shape, np.array(arr.strides) // arr.itemsize)):
            t.shape[i], t.stride[i] = s, int(st)
        t.dtype = _C.GT_F32 if dtype is None else dtype
        return t

    q = np.zeros((1, 2, 4, 8), np.float32)

    def call(qq=q, kk=q, kr=q, mode=0, n_dims=8, n_pos_q=4, n_pos_k=4, qd=None):
        tq, tk, tkr, to = t4(qq, qd), t4(kk, qd), t4(kr, qd), t4(q.copy(), qd)
        pos = np.arange(8, dtype=np.int32)
        rc = _C.lib.gtb_sdpa_fwd_rope(ctypes.byref(tq), ctypes.byref(tk), ctypes.byref(tk), None, 0.0, 1,
                                      pos.ctypes.data, n_pos_q, pos.ctypes.data, n_pos_k, n_dims, mode, 10000.0, 1.0,
                                      1, ctypes.byref(tkr), ctypes.byref(to), None, None)
        return rc, _C.lib.gtb_last_error().decode()

    rc, msg = call(kk=np.zeros((1, 3, 4, 8), np.float32), kr=np.zeros((1, 3, 4, 8), np.float32))
    assert rc != 0 and "num_heads must be divisible by num_kv_heads" in msg
    rc, msg = call(mode=1)
    assert rc != 0 and "mode must be 0 (normal) or 2 (NeoX)" in msg
    rc, msg = call(n_dims=10)
    assert rc != 0 and "n_dims must be an even number" in msg
    rc, msg = call(n_pos_q=3)
    assert rc != 0 and "a position for each of the 4 queries" in msg
    rc, msg = call(kr=np.zeros((1, 2, 4, 4), np.float32))
    assert rc != 0 and "k_rot" in msg
    rc, msg = call(qd=_C.GT_F64)
    assert rc != 0 and "f32, f16 or bf16" in msg
    rc, msg = call()  # well-formed, but host memory: the engine has no CPU path
    assert rc != 0 and "no CPU path" in msg
