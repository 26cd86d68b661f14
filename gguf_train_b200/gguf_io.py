"""GGUF files for the decode path: Q8_0 KV caches (and float tensors) to and from disk.

The reference reads and writes GGUF with `load_gguf` / `save_gguf` (gguf_train/gguf/__init__.py:133-300);
this module keeps those names and their main arguments for the tensors the attention path uses. The
layout is GGUF version 3 as published with ggml: the magic "GGUF", the version, the tensor and
key/value counts, typed key/value pairs, one info record per tensor (name, dims innermost first, ggml
type, offset into the data section), then the data section, every tensor starting on a multiple of
`general.alignment` (32 unless the file says otherwise).

A Q8_0 tensor of logical shape (..., D) is stored as ggml stores it: D/32 blocks of 34 bytes per row
(fp16 scale, 32 int8), exactly the uint8 (..., D/32*34) blocks that `quantize_q8_0`, `q8_0_append`
and `decode_q8_0` use, so a cache goes from disk to the decode kernel without conversion. Here such a
tensor is a `Q8_0` wrapper around its blocks. File I/O runs on the host; tensors are placed on the
device the caller names, and dequantisation (optional) runs on the GPU.

GGUF holds at most four dimensions and no uint8, bool or complex element type. As the reference's writer
does (csrc/gt_ops_extra.cpp:1497-1516, :1785-1788), such tensors are stored in a form GGUF can hold -- the
outer dimensions beyond four folded into the fourth, a scalar as one element, uint8/bool as int8 bytes,
complex as (real, imaginary) float pairs in an extra innermost dimension -- and what that loses is kept
under two reserved keys, written only when needed: `gguf_train.shape.<name>` (int64 array, the real
shape) and `gguf_train.dtype.<name>` (string: "uint8", "bool", "complex64", "complex128"). The reader
applies them (gt_ops_extra.cpp:1853-1905) and leaves them out of the metadata it returns
(gguf_train/gguf/__init__.py:84-85), so files written by either side read back the same on the other.
"""

from __future__ import annotations

import struct
from pathlib import Path
from typing import NamedTuple

import numpy as np
import torch

_MAGIC = b"GGUF"
_VERSION = 3
_ALIGN = 32

# ggml tensor types handled here: id -> (values per block, bytes per block, numpy dtype of a value)
_Q8_0 = 8
_TYPES = {0: (1, 4, np.float32), 1: (1, 2, np.float16), 30: (1, 2, None), _Q8_0: (32, 34, None),
          24: (1, 1, np.int8), 25: (1, 2, np.int16), 26: (1, 4, np.int32), 27: (1, 8, np.int64), 28: (1, 8, np.float64)}
_TORCH_TYPE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 30, torch.int8: 24, torch.int16: 25,
               torch.int32: 26, torch.int64: 27, torch.float64: 28}

# GGUF metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f", _BOOL: "<?",
           _U64: "<Q", _I64: "<q", _F64: "<d"}


_SHAPE_KEY = "gguf_train.shape."
_DTYPE_KEY = "gguf_train.dtype."
_RESERVED = (_SHAPE_KEY, _DTYPE_KEY)
_MAX_DIMS = 4
# element types GGUF cannot name: torch dtype -> (recorded name, carrier ggml type, values per element)
_RECORDED = {torch.uint8: ("uint8", 24, 1), torch.bool: ("bool", 24, 1),
             torch.complex64: ("complex64", 0, 2), torch.complex128: ("complex128", 28, 2)}
_FROM_RECORDED = {name: (dt, carrier, per) for dt, (name, carrier, per) in _RECORDED.items()}


class Q8_0(NamedTuple):
    """A Q8_0 tensor: `blocks` is uint8 (..., D/32*34), the layout of quantize_q8_0."""
    blocks: torch.Tensor


class GGUFFile:
    """An opened GGUF file: `metadata` (key -> int, float, bool, str or a list of those) and
    `tensors` (name -> torch tensor, or Q8_0 for quantised ones), as the reference's GGUFFile."""

    def __init__(self, path, dequantize: bool = False, device=None):
        self.path = Path(path)
        meta, infos, data_start = _read_header(self.path)
        self.metadata = {k: v for k, v in meta.items() if not k.startswith(_RESERVED)}
        self.tensors = {}
        raw = np.memmap(self.path, dtype=np.uint8, mode="r")
        dev = torch.device(device) if device is not None else torch.device("cpu")
        for name, shape, ggml_type, offset in infos:
            per_block, block_bytes, _ = _TYPES[ggml_type]
            n = int(np.prod(shape, dtype=np.int64)) if shape else 1
            nbytes = n // per_block * block_bytes
            start = data_start + offset
            if start + nbytes > raw.size:
                raise ValueError(f"load_gguf: tensor {name!r} runs past the end of {self.path}")
            buf = np.array(raw[start:start + nbytes])
            recorded = meta.get(_DTYPE_KEY + name)
            if recorded is not None:
                self.tensors[name] = _recorded_to_torch(buf, shape, ggml_type, recorded,
                                                        meta.get(_SHAPE_KEY + name), dev, name)
                continue
            t = _to_torch(buf, _natural_shape(shape) if _SHAPE_KEY + name in meta else shape,
                          ggml_type, dev, dequantize, name)
            if _SHAPE_KEY + name in meta:
                t = _reshape_recorded(t, meta[_SHAPE_KEY + name], name)
            self.tensors[name] = t
        del raw

    def __getitem__(self, name):
        return self.tensors[name]

    def keys(self):
        return self.tensors.keys()


def load_gguf(path, dequantize: bool = False, return_metadata: bool = False, device=None):
    """Load a .gguf file: returns a GGUFFile, or (tensors, metadata) with `return_metadata`. Tensors
    go to `device` (default: host memory). Q8_0 tensors come back as Q8_0 blocks, ready for
    decode_q8_0 once on a CUDA device; with `dequantize` they become float32 on that device (the
    dequantisation runs on the GPU, so it needs a CUDA `device`)."""
    gf = GGUFFile(path, dequantize=dequantize, device=device)
    if return_metadata:
        return gf.tensors, gf.metadata
    return gf


def save_gguf(path, tensors: dict, metadata: dict | None = None) -> None:
    """Write `tensors` (name -> torch tensor or numpy array of f32/f16/bf16/f64/int8-64, or Q8_0) and
    `metadata` (name -> bool, int, float, str, or a list of one of those) as a GGUF v3 file."""
    meta = dict(metadata or {})
    for key in meta:
        if str(key).startswith(_RESERVED):
            raise ValueError(f"save_gguf: metadata key {key!r} is reserved: gguf_train.shape.* and "
                             "gguf_train.dtype.* describe how tensors are stored")
    align = int(meta.get("general.alignment", _ALIGN))
    if align <= 0 or align % 8:
        raise ValueError("save_gguf: general.alignment must be a positive multiple of 8")
    records, blobs = [], []
    offset = 0
    recorded = {}
    for name, t in tensors.items():
        ggml_type, shape, data, real_shape, dtype_name = _from_value(name, t)
        if real_shape is not None:
            recorded[_SHAPE_KEY + name] = _I64, list(real_shape)
        if dtype_name is not None:
            recorded[_DTYPE_KEY + name] = _STR, dtype_name
        records.append((name, shape, ggml_type, offset))
        blobs.append(data)
        offset += _pad(len(data), align)
    out = bytearray()
    out += _MAGIC + struct.pack("<IQQ", _VERSION, len(records), len(meta) + len(recorded))
    for key, value in meta.items():
        out += _string(key)
        out += _value(key, value)
    for key, (t, value) in recorded.items():
        out += _string(key)
        if t == _STR:
            out += struct.pack("<I", _STR) + _string(value)
        else:
            out += struct.pack("<IIQ", _ARR, _I64, len(value)) + b"".join(struct.pack("<q", d) for d in value)
    for name, shape, ggml_type, off in records:
        out += _string(name)
        out += struct.pack("<I", len(shape))
        for d in reversed(shape):  # innermost first
            out += struct.pack("<Q", d)
        out += struct.pack("<IQ", ggml_type, off)
    out += b"\0" * (_pad(len(out), align) - len(out))
    with open(path, "wb") as f:
        f.write(out)
        for data in blobs:
            f.write(data)
            f.write(b"\0" * (_pad(len(data), align) - len(data)))


# ------------------------------------------------------------------ writing

def _pad(n: int, align: int) -> int:
    return (n + align - 1) // align * align


def _string(s) -> bytes:
    raw = s if isinstance(s, (bytes, bytearray)) else str(s).encode("utf-8")
    return struct.pack("<Q", len(raw)) + bytes(raw)


def _scalar_type(key, v) -> int:
    if isinstance(v, bool):
        return _BOOL
    if isinstance(v, (int, np.integer)):
        if -(1 << 63) <= int(v) < (1 << 63):
            return _I64
        if 0 <= int(v) < (1 << 64):
            return _U64
        raise ValueError(f"save_gguf: metadata {key!r} does not fit in 64 bits")
    if isinstance(v, (float, np.floating)):
        return _F64
    if isinstance(v, (str, bytes, bytearray)):
        return _STR
    raise ValueError(f"save_gguf: metadata {key!r} has unsupported type {type(v).__name__}")


def _scalar(t: int, v) -> bytes:
    return _string(v) if t == _STR else struct.pack(_SCALAR[t], v)


def _value(key, v) -> bytes:
    if key == "general.alignment":
        return struct.pack("<I", _U32) + struct.pack("<I", int(v))
    if isinstance(v, (list, tuple)):
        types = {_scalar_type(key, e) for e in v} or {_I64}
        if types == {_I64, _F64}:
            types = {_F64}
        if len(types) != 1:
            raise ValueError(f"save_gguf: metadata list {key!r} mixes value types")
        t = types.pop()
        return struct.pack("<IIQ", _ARR, t, len(v)) + b"".join(_scalar(t, e) for e in v)
    t = _scalar_type(key, v)
    return struct.pack("<I", t) + _scalar(t, v)


def _stored_shape(shape, per_block: int = 1):
    """The dimensions GGUF keeps for a tensor of logical `shape` (outermost first, at most four), and
    whether a reader would need the recorded shape to get `shape` back. Mirrors the reference's plan
    (gt_ops_extra.cpp:1571-1594): a scalar is one element, an empty tensor is zero elements, a
    quantised tensor whose rows are not whole blocks is one row, and dimensions beyond four fold into
    the outermost one kept."""
    shape = tuple(int(d) for d in shape)
    count = int(np.prod(shape, dtype=np.int64)) if shape else 1
    if count == 0:
        stored = (0,)
    elif not shape:
        stored = (1,)
    elif per_block > 1 and shape[-1] % per_block:
        stored = (count,)
    elif len(shape) > _MAX_DIMS:
        outer = int(np.prod(shape[:len(shape) - _MAX_DIMS + 1], dtype=np.int64))
        stored = (outer,) + shape[len(shape) - _MAX_DIMS + 1:]
    else:
        stored = shape
    return stored, _natural_shape(stored) != shape


def _natural_shape(stored):
    """The shape a reader derives from stored dimensions alone: trailing (outermost) ones dropped,
    at least one dimension kept (gt_ops_extra.cpp:1534-1547)."""
    dims = list(stored) or [1]
    while len(dims) > 1 and dims[0] == 1:
        dims.pop(0)
    return tuple(dims)


def _from_value(name, t):
    """(ggml type, stored shape, bytes, recorded shape or None, recorded dtype name or None) of a
    tensor to write."""
    if isinstance(t, Q8_0):
        b = t.blocks.detach().to("cpu").contiguous()
        if b.dtype != torch.uint8 or b.ndim < 1 or b.shape[-1] % 34:
            raise ValueError(f"save_gguf: Q8_0 tensor {name!r} must be uint8 blocks (..., D/32*34)")
        shape = tuple(b.shape[:-1]) + (b.shape[-1] // 34 * 32,)
        stored, need = _stored_shape(shape, 32)
        return _Q8_0, stored, b.numpy().tobytes(), shape if need else None, None
    if isinstance(t, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(t))
    if not isinstance(t, torch.Tensor) or (t.dtype not in _TORCH_TYPE and t.dtype not in _RECORDED):
        raise ValueError(f"save_gguf: tensor {name!r} must be a float, integer, uint8, bool or complex "
                         "tensor, or Q8_0 blocks")
    c = t.detach().to("cpu").contiguous()
    shape = tuple(c.shape)
    if c.dtype in _RECORDED:
        dtype_name, ggml_type, per = _RECORDED[c.dtype]
        if per == 2:
            raw = torch.view_as_real(c)
        else:
            raw = c.view(torch.int8) if c.dtype == torch.uint8 else c.to(torch.int8)
        stored, need = _stored_shape(tuple(raw.shape))
        # a complex tensor's natural shape is its stored one without the (real, imaginary) pair
        natural = _natural_shape(stored)
        natural = natural[:-1] if per == 2 and natural and natural[-1] == 2 else (() if per == 2 else natural)
        real = shape if natural != shape else None
        return ggml_type, stored, raw.numpy().tobytes(), real, dtype_name
    raw = c.view(torch.int16) if c.dtype == torch.bfloat16 else c
    stored, need = _stored_shape(shape)
    return _TORCH_TYPE[c.dtype], stored, raw.numpy().tobytes(), shape if need else None, None


# ------------------------------------------------------------------ reading

class _Cursor:
    def __init__(self, f):
        self.f = f

    def take(self, fmt: str):
        size = struct.calcsize(fmt)
        raw = self.f.read(size)
        if len(raw) != size:
            raise ValueError("load_gguf: the file ends inside its header")
        return struct.unpack(fmt, raw)

    def string(self) -> str:
        (n,) = self.take("<Q")
        raw = self.f.read(n)
        if len(raw) != n:
            raise ValueError("load_gguf: the file ends inside its header")
        return raw.decode("utf-8", errors="replace")

    def value(self, t: int):
        if t == _STR:
            return self.string()
        if t == _ARR:
            et, n = self.take("<IQ")
            return [self.value(et) for _ in range(n)]
        if t not in _SCALAR:
            raise ValueError(f"load_gguf: unknown metadata value type {t}")
        return self.take(_SCALAR[t])[0]


def _read_header(path: Path):
    with open(path, "rb") as f:
        if f.read(4) != _MAGIC:
            raise ValueError(f"load_gguf: {path} is not a GGUF file")
        c = _Cursor(f)
        (version,) = c.take("<I")
        if version not in (2, 3):
            raise ValueError(f"load_gguf: GGUF version {version} is not supported (2 or 3)")
        n_tensors, n_kv = c.take("<QQ")
        meta = {}
        for _ in range(n_kv):
            key = c.string()
            (t,) = c.take("<I")
            meta[key] = c.value(t)
        infos = []
        for _ in range(n_tensors):
            name = c.string()
            (nd,) = c.take("<I")
            ne = c.take("<" + "Q" * nd) if nd else ()
            ggml_type, offset = c.take("<IQ")
            if ggml_type not in _TYPES:
                raise ValueError(f"load_gguf: tensor {name!r} has ggml type {ggml_type}, which this engine does not read")
            infos.append((name, tuple(int(d) for d in reversed(ne)), ggml_type, offset))
        data_start = _pad(f.tell(), int(meta.get("general.alignment", _ALIGN)))
    return meta, infos, data_start


def _to_torch(buf: np.ndarray, shape, ggml_type: int, dev: torch.device, dequantize: bool, name: str):
    if ggml_type == _Q8_0:
        if shape and shape[-1] % 32:
            raise ValueError(f"load_gguf: Q8_0 tensor {name!r} has rows of {shape[-1]} values (not whole blocks)")
        blocks = torch.from_numpy(buf).reshape(tuple(shape[:-1]) + (shape[-1] // 32 * 34,)).to(dev)
        if not dequantize:
            return Q8_0(blocks)
        if dev.type != "cuda":
            raise RuntimeError("load_gguf: dequantize runs on the GPU; give a CUDA device")
        from .functional import dequantize_q8_0

        return dequantize_q8_0(blocks, torch.float32)
    if ggml_type == 30:
        return torch.from_numpy(buf.view(np.int16).copy()).view(torch.bfloat16).reshape(shape).to(dev)
    return torch.from_numpy(buf.view(_TYPES[ggml_type][2]).copy()).reshape(shape).to(dev)


def _reshape_recorded(t, shape, name: str):
    """Apply a recorded `gguf_train.shape.<name>` to a tensor read with its stored dimensions."""
    if not isinstance(shape, list) or not all(isinstance(d, int) and d >= 0 for d in shape):
        raise ValueError(f"load_gguf: tensor {name!r}: the recorded shape is not an int64 array")
    shape = tuple(shape)
    if isinstance(t, Q8_0):
        if not shape or shape[-1] % 32:
            raise ValueError(f"load_gguf: Q8_0 tensor {name!r}: recorded shape {shape} is not whole blocks")
        want = shape[:-1] + (shape[-1] // 32 * 34,)
        if int(np.prod(want, dtype=np.int64)) != t.blocks.numel():
            raise ValueError(f"load_gguf: tensor {name!r}: the shape does not match the stored elements")
        return Q8_0(t.blocks.reshape(want))
    if int(np.prod(shape, dtype=np.int64)) != t.numel():
        raise ValueError(f"load_gguf: tensor {name!r}: the shape does not match the {t.numel()} stored elements")
    return t.reshape(shape)


def _recorded_to_torch(buf: np.ndarray, stored, ggml_type: int, dtype_name, shape, dev, name: str):
    """A tensor whose element type GGUF could not name, from its carrier bytes and the recorded
    `gguf_train.dtype.<name>` (and shape, when one was recorded)."""
    if dtype_name not in _FROM_RECORDED:
        raise ValueError(f"load_gguf: tensor {name!r}: unknown recorded dtype {dtype_name!r}")
    dt, carrier, per = _FROM_RECORDED[dtype_name]
    if carrier != ggml_type:
        raise ValueError(f"load_gguf: tensor {name!r}: recorded as {dtype_name} but stored as ggml type {ggml_type}")
    vals = torch.from_numpy(buf.view(_TYPES[ggml_type][2]).copy())
    if per == 2:
        if vals.numel() % 2:
            raise ValueError(f"load_gguf: tensor {name!r}: a complex tensor needs an even number of stored values")
        t = torch.view_as_complex(vals.reshape(-1, 2))
        natural = _natural_shape(stored)
        natural = natural[:-1] if natural and natural[-1] == 2 else ()
    else:
        t = vals.view(torch.uint8) if dt == torch.uint8 else vals != 0
        natural = _natural_shape(stored)
    t = _reshape_recorded(t, list(shape) if shape is not None else list(natural), name)
    return t.to(dev)
