"""safetensors-format container of a repacked engine (DeviceEngine.save_repacked /
from_repacked): an 8-byte little-endian header length, a JSON header mapping each tensor name
to {"dtype", "shape", "data_offsets"} plus "__metadata__", padded with spaces to a multiple of
8 bytes, then the tensors' bytes back to back. Host-side only (no device access)."""

from __future__ import annotations

import json
import struct

FORMAT = "pulsar_b200.arena.v1"
_ITEM = {"BF16": 2, "F32": 4}


def write(path: str, tensors, metadata: dict) -> None:
    """tensors: iterable of (name, dtype "BF16" | "F32", shape list, bytes)."""
    header, blobs, off = {}, [], 0
    for name, dtype, shape, b in tensors:
        n = 1
        for d in shape:
            n *= int(d)
        if dtype not in _ITEM or n * _ITEM[dtype] != len(b):
            raise ValueError(f"{name}: {len(b)} bytes do not hold {dtype} {list(shape)}")
        header[name] = {"dtype": dtype, "shape": [int(d) for d in shape], "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    hj = json.dumps(header).encode()
    hj += b" " * (-len(hj) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for b in blobs:
            f.write(b)


def read(path: str):
    """(header without "__metadata__", metadata, data bytes after the header); checks that the
    offsets tile the data and that the file is a repacked pulsar_b200 arena."""
    with open(path, "rb") as f:
        (hl,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hl))
        data = f.read()
    meta = header.pop("__metadata__", {})
    if meta.get("format") != FORMAT:
        raise ValueError(f"{path}: not a pulsar_b200 repacked arena (format {meta.get('format')!r})")
    end = 0
    for name, h in sorted(header.items(), key=lambda kv: kv[1]["data_offsets"][0]):
        if h.get("dtype") not in _ITEM:
            raise ValueError(f"{path}: tensor {name} has dtype {h.get('dtype')!r}; a repacked arena holds only "
                             f"{', '.join(sorted(_ITEM))}")
        b0, b1 = h["data_offsets"]
        n = 1
        for d in h["shape"]:
            n *= int(d)
        if b0 != end or b1 - b0 != n * _ITEM[h["dtype"]]:
            raise ValueError(f"{path}: tensor {name} has inconsistent offsets")
        end = b1
    if end != len(data):
        raise ValueError(f"{path}: {len(data) - end} trailing or missing bytes")
    return header, meta, data
