"""GGUF I/O of the decode path (gguf_train_b200.gguf_io) on the host, pinned against gguf-py, ggml's
own Python GGUF package: files this module writes read back in gguf-py with the same metadata, shapes,
types and bytes, and files gguf-py writes (Q8_0 from its quantiser) load here to the same blocks that
the engine's quantiser and the oracle produce. The reference's own tests round-trip its
save_gguf/load_gguf the same way (tests/test_gguf_and_llama.py:44, tests/test_gguf_roundtrip.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle as O


def _blocks(x: np.ndarray) -> torch.Tensor:
    q = O.q8_0_quantize(x.reshape(-1, x.shape[-1]))
    return torch.from_numpy(q.reshape(x.shape[:-1] + (x.shape[-1] // 32 * 34,)))


def test_written_files_read_back_in_gguf_py(tmp_path):
    from gguf import GGMLQuantizationType, GGUFReader

    from gguf_train_b200 import gguf_io

    rs = np.random.RandomState(1)
    k = rs.randn(2, 3, 10, 64).astype(np.float32)
    tensors = {
        "cache.k": gguf_io.Q8_0(_blocks(k)),
        "w.f32": torch.from_numpy(rs.randn(4, 5).astype(np.float32)),
        "w.f16": torch.from_numpy(rs.randn(7).astype(np.float16)),
        "w.bf16": torch.randn(3, 8).to(torch.bfloat16),
        "lens": torch.tensor([10, 3], dtype=torch.int32),
    }
    meta = {"general.name": "kv cache", "seq.count": 2, "rope.freq_base": 10000.0, "flag": True,
            "lens.list": [10, 3], "names": ["a", "b"]}
    path = tmp_path / "cache.gguf"
    gguf_io.save_gguf(path, tensors, meta)

    r = GGUFReader(path)
    assert r.fields["general.name"].contents() == "kv cache"
    assert r.fields["seq.count"].contents() == 2
    assert r.fields["rope.freq_base"].contents() == 10000.0
    assert r.fields["flag"].contents() is True
    assert r.fields["lens.list"].contents() == [10, 3]
    assert r.fields["names"].contents() == ["a", "b"]
    by_name = {t.name: t for t in r.tensors}
    t = by_name["cache.k"]
    assert t.tensor_type == GGMLQuantizationType.Q8_0
    assert [int(d) for d in t.shape] == [64, 10, 3, 2]  # innermost first
    assert np.asarray(t.data).tobytes() == tensors["cache.k"].blocks.numpy().tobytes()
    assert by_name["w.f32"].tensor_type == GGMLQuantizationType.F32
    assert np.array_equal(np.asarray(by_name["w.f32"].data).reshape(4, 5), tensors["w.f32"].numpy())
    assert by_name["w.f16"].tensor_type == GGMLQuantizationType.F16
    assert by_name["w.bf16"].tensor_type == GGMLQuantizationType.BF16
    assert np.asarray(by_name["w.bf16"].data).tobytes() == tensors["w.bf16"].view(torch.int16).numpy().tobytes()
    assert by_name["lens"].tensor_type == GGMLQuantizationType.I32


def test_gguf_py_files_load_to_the_engines_blocks(tmp_path):
    import gguf
    from gguf import GGMLQuantizationType, GGUFWriter

    from gguf_train_b200 import gguf_io

    rs = np.random.RandomState(2)
    k = (rs.randn(2, 4, 12, 128) * 2).astype(np.float32)
    qk = gguf.quants.quantize(k.reshape(-1, 128), GGMLQuantizationType.Q8_0).reshape(2, 4, 12, 4 * 34)
    path = tmp_path / "from_gguf_py.gguf"
    w = GGUFWriter(path, arch="llama")
    w.add_uint32("cache.max_len", 12)
    w.add_string("cache.note", "written by gguf-py")
    w.add_tensor("blk.0.attn_k.cache", qk, raw_dtype=GGMLQuantizationType.Q8_0)
    w.add_tensor("norm", rs.randn(128).astype(np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()

    tensors, meta = gguf_io.load_gguf(path, return_metadata=True)
    assert meta["general.architecture"] == "llama"
    assert meta["cache.max_len"] == 12 and meta["cache.note"] == "written by gguf-py"
    kc = tensors["blk.0.attn_k.cache"]
    assert isinstance(kc, gguf_io.Q8_0) and tuple(kc.blocks.shape) == (2, 4, 12, 136)
    assert np.array_equal(kc.blocks.numpy(), qk)
    assert np.array_equal(kc.blocks.numpy(), _blocks(k).numpy())  # the engine's quantiser, restated
    assert tensors["norm"].dtype == torch.float32 and tensors["norm"].shape == (128,)


def test_round_trip_and_alignment(tmp_path):
    from gguf_train_b200 import gguf_io

    rs = np.random.RandomState(3)
    v = rs.randn(1, 2, 5, 32).astype(np.float32)
    src = {"v": gguf_io.Q8_0(_blocks(v)), "x": torch.randn(3, 3, dtype=torch.float64),
           "b": torch.randn(9).to(torch.bfloat16)}
    path = tmp_path / "rt.gguf"
    gguf_io.save_gguf(path, src, {"general.alignment": 64, "k": -5})
    gf = gguf_io.load_gguf(path)
    assert gf.metadata["general.alignment"] == 64 and gf.metadata["k"] == -5
    assert torch.equal(gf["v"].blocks, src["v"].blocks)
    assert torch.equal(gf["x"], src["x"]) and torch.equal(gf["b"], src["b"])
    raw = path.read_bytes()
    assert raw[:4] == b"GGUF" and len(raw) % 64 == 0


def test_errors(tmp_path):
    from gguf_train_b200 import gguf_io

    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"NOPE" + bytes(20))
    with pytest.raises(ValueError, match="not a GGUF file"):
        gguf_io.load_gguf(bad)
    with pytest.raises(ValueError, match="must be uint8 blocks"):
        gguf_io.save_gguf(tmp_path / "x.gguf", {"q": gguf_io.Q8_0(torch.zeros(3, 33, dtype=torch.uint8))})
    with pytest.raises(ValueError, match="unsupported type"):
        gguf_io.save_gguf(tmp_path / "y.gguf", {}, {"d": {"nested": 1}})
    gguf_io.save_gguf(tmp_path / "z.gguf", {"q": gguf_io.Q8_0(torch.zeros(1, 34, dtype=torch.uint8))})
    with pytest.raises(RuntimeError, match="dequantize runs on the GPU"):
        gguf_io.load_gguf(tmp_path / "z.gguf", dequantize=True)


def test_shapes_and_types_gguf_cannot_hold_round_trip(tmp_path):
    """More than four dimensions, scalars, leading ones, empty tensors, uint8, bool and complex: stored
    in a form GGUF holds (at most four dimensions, int8/f32/f64 carriers) with the real shape and type
    under the reserved keys, as the reference writes them (csrc/gt_ops_extra.cpp:1497-1516); gguf-py
    still reads the file, and the reserved keys stay out of the metadata."""
    from gguf import GGUFReader

    from gguf_train_b200 import gguf_io

    rs = np.random.RandomState(5)
    k = rs.randn(2, 1, 3, 2, 4, 32).astype(np.float32)
    src = {
        "five": torch.from_numpy(rs.randn(2, 3, 1, 4, 5).astype(np.float32)),
        "scalar": torch.tensor(3.5, dtype=torch.float64),
        "lead": torch.from_numpy(rs.randn(1, 5).astype(np.float32)),
        "empty": torch.zeros(0, 4, dtype=torch.float16),
        "u8": torch.arange(250, 256, dtype=torch.uint8).reshape(2, 3),
        "mask": torch.tensor([[True, False, True], [False, False, True]]),
        "c64": torch.randn(3, 2, dtype=torch.complex64),
        "c128": torch.tensor(1 - 2j, dtype=torch.complex128),
        "q6": gguf_io.Q8_0(_blocks(k)),
        "plain": torch.from_numpy(rs.randn(2, 3, 4, 5).astype(np.float32)),
    }
    path = tmp_path / "odd.gguf"
    gguf_io.save_gguf(path, src, {"general.name": "odd"})

    r = GGUFReader(path)
    assert all(len(t.shape) <= 4 for t in r.tensors)
    keys = set(r.fields)
    assert "gguf_train.shape.five" in keys and "gguf_train.dtype.u8" in keys
    assert "gguf_train.shape.plain" not in keys and "gguf_train.dtype.plain" not in keys

    gf = gguf_io.load_gguf(path)
    assert not any(k.startswith("gguf_train.") for k in gf.metadata)
    for name, t in src.items():
        got = gf[name]
        if isinstance(t, gguf_io.Q8_0):
            assert got.blocks.shape == t.blocks.shape and torch.equal(got.blocks, t.blocks)
        else:
            assert got.dtype == t.dtype and got.shape == t.shape, name
            assert torch.equal(got, t), name

    with pytest.raises(ValueError, match="is reserved"):
        gguf_io.save_gguf(tmp_path / "r.gguf", {}, {"gguf_train.shape.x": [1]})


def test_reserved_keys_written_by_another_writer_are_applied(tmp_path):
    """A file laid out as the reference writes a 5-D uint8 tensor (int8 bytes, the outer dimensions
    folded, real shape and type under the reserved keys), produced here with gguf-py, loads with its
    real shape and type."""
    from gguf import GGMLQuantizationType, GGUFWriter

    from gguf_train_b200 import gguf_io

    real = (2, 2, 3, 1, 4)
    vals = np.arange(48, dtype=np.uint8) * 5
    path = tmp_path / "ref_like.gguf"
    w = GGUFWriter(path, arch="llama")
    w.add_array("gguf_train.shape.t", list(real))
    w.add_string("gguf_train.dtype.t", "uint8")
    w.add_tensor("t", vals.view(np.int8).reshape(4, 3, 1, 4), raw_dtype=GGMLQuantizationType.I8)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    gf = gguf_io.load_gguf(path)
    assert gf["t"].dtype == torch.uint8 and tuple(gf["t"].shape) == real
    assert torch.equal(gf["t"].flatten(), torch.from_numpy(vals))
