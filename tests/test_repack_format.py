"""The safetensors-format container of repacked engines (pulsar_b200.repack), on the CPU."""

from __future__ import annotations

import json
import struct

import numpy as np
import pytest

from pulsar_b200 import repack


def test_roundtrip_layout_and_metadata(tmp_path):
    a = np.arange(10, dtype=np.uint16)                       # bf16 bit patterns
    b = np.linspace(-1, 1, 6, dtype=np.float32).reshape(2, 3)
    p = str(tmp_path / "x.safetensors")
    repack.write(p, [("arena.tok_emb", "BF16", [10], a.tobytes()), ("core.0.x", "F32", [2, 3], b.tobytes())],
                 {"format": repack.FORMAT, "config": json.dumps({"d_model": 1024})})
    raw = open(p, "rb").read()
    (hl,) = struct.unpack("<Q", raw[:8])
    assert hl % 8 == 0
    header, meta, data = repack.read(p)
    assert meta["format"] == repack.FORMAT and json.loads(meta["config"]) == {"d_model": 1024}
    assert header["arena.tok_emb"] == {"dtype": "BF16", "shape": [10], "data_offsets": [0, 20]}
    assert header["core.0.x"]["data_offsets"] == [20, 44]
    assert np.array_equal(np.frombuffer(data, np.uint16, 10, 0), a)
    assert np.array_equal(np.frombuffer(data, np.float32, 6, 20).reshape(2, 3), b)


def test_rejects_size_mismatch_and_foreign_files(tmp_path):
    with pytest.raises(ValueError, match="do not hold"):
        repack.write(str(tmp_path / "y"), [("t", "F32", [3], bytes(8))], {"format": repack.FORMAT})
    p = tmp_path / "z.safetensors"
    h = json.dumps({"__metadata__": {"format": "other"}}).encode()
    p.write_bytes(struct.pack("<Q", len(h)) + h)
    with pytest.raises(ValueError, match="not a pulsar_b200 repacked arena"):
        repack.read(str(p))
    p2 = str(tmp_path / "w.safetensors")
    repack.write(p2, [("t", "F32", [2], np.zeros(2, np.float32).tobytes())], {"format": repack.FORMAT})
    with open(p2, "ab") as f:
        f.write(b"junk")
    with pytest.raises(ValueError, match="trailing"):
        repack.read(p2)


def test_rejects_foreign_dtype(tmp_path):
    """A file with our format tag but a dtype the arena never holds fails validation with a
    ValueError naming the tensor (not a bare KeyError)."""
    p = tmp_path / "f16.safetensors"
    h = json.dumps({"__metadata__": {"format": repack.FORMAT},
                    "t": {"dtype": "F16", "shape": [2], "data_offsets": [0, 4]}}).encode()
    h += b" " * (-len(h) % 8)
    p.write_bytes(struct.pack("<Q", len(h)) + h + bytes(4))
    with pytest.raises(ValueError, match="tensor t has dtype 'F16'"):
        repack.read(str(p))
