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


class Q8_0(NamedTuple):
    """A Q8_0 tensor: `blocks` is uint8 (..., D/32*34), the layout of quantize_q8_0."""
    blocks: torch.Tensor


class GGUFFile:
    """An opened GGUF file: `metadata` (key -> int, float, bool, str or a list of those) and
    `tensors` (name -> torch tensor, or Q8_0 for quantised ones), as the reference's GGUFFile."""

    def __init__(self, path, dequantize: bool = False, device=None):
        self.path = Path(path)
        self.metadata, infos, data_start = _read_header(self.path)
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
            self.tensors[name] = _to_torch(buf, shape, ggml_type, dev, dequantize, name)
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
    align = int(meta.get("general.alignment", _ALIGN))
    if align <= 0 or align % 8:
        raise ValueError("save_gguf: general.alignment must be a positive multiple of 8")
    records, blobs = [], []
    offset = 0
    for name, t in tensors.items():
        ggml_type, shape, data = _from_value(name, t)
        records.append((name, shape, ggml_type, offset))
        blobs.append(data)
        offset += _pad(len(data), align)
    out = bytearray()
    out += _MAGIC + struct.pack("<IQQ", _VERSION, len(records), len(meta))
    for key, value in meta.items():
        out += _string(key)
        out += _value(key, value)
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


def _from_value(name, t):
    """(ggml type, logical shape, bytes) of a tensor to write."""
    if isinstance(t, Q8_0):
        b = t.blocks.detach().to("cpu").contiguous()
        if b.dtype != torch.uint8 or b.ndim < 1 or b.shape[-1] % 34:
            raise ValueError(f"save_gguf: Q8_0 tensor {name!r} must be uint8 blocks (..., D/32*34)")
        shape = tuple(b.shape[:-1]) + (b.shape[-1] // 34 * 32,)
        return _Q8_0, shape, b.numpy().tobytes()
    if isinstance(t, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(t))
    if not isinstance(t, torch.Tensor) or t.dtype not in _TORCH_TYPE:
        raise ValueError(f"save_gguf: tensor {name!r} must be a float or integer tensor, or Q8_0 blocks")
    c = t.detach().to("cpu").contiguous()
    raw = c.view(torch.int16) if c.dtype == torch.bfloat16 else c
    return _TORCH_TYPE[t.dtype], tuple(t.shape), raw.numpy().tobytes()


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
