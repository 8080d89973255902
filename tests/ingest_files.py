"""Writers of small GGUF and safetensors files for the ingest tests (test
infrastructure: the product only reads these formats).  They follow the
published layouts: GGUF v3 (magic, version, tensor and metadata counts,
typed metadata, tensor table with GGUF-order dims, aligned data section) and
safetensors (8-byte header length, JSON header, raw data)."""
from __future__ import annotations

import json
import struct

import numpy as np


def _s(b: bytearray, text: str) -> None:
    e = text.encode()
    b += struct.pack("<Q", len(e)) + e


def write_gguf(path, tensors, metadata=None, alignment: int = 32) -> None:
    """tensors: list of (name, dims in GGUF order, ggml type, raw bytes)."""
    metadata = dict(metadata or {})
    if alignment != 32:
        metadata["general.alignment"] = ("u32", alignment)
    b = bytearray(struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(metadata)))
    for k, (kind, v) in metadata.items():
        _s(b, k)
        if kind == "str":
            b += struct.pack("<I", 8)
            _s(b, v)
        elif kind == "u32":
            b += struct.pack("<II", 4, v)
        elif kind == "f32":
            b += struct.pack("<If", 6, v)
        elif kind == "arr_u32":
            b += struct.pack("<IIQ", 9, 4, len(v)) + b"".join(struct.pack("<I", x) for x in v)
        else:
            raise ValueError(kind)
    off = 0
    offs = []
    for name, dims, t, data in tensors:
        _s(b, name)
        b += struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        b += struct.pack("<IQ", t, off)
        offs.append(off)
        off = (off + len(data) + alignment - 1) // alignment * alignment
    pad = (-len(b)) % alignment
    b += b"\0" * pad
    base = len(b)
    out = bytearray(b)
    for (name, dims, t, data), o in zip(tensors, offs):
        need = base + o - len(out)
        out += b"\0" * need
        out += bytes(data)
    with open(path, "wb") as f:
        f.write(out)


def write_safetensors(path, tensors: dict) -> None:
    """tensors: name -> (dtype string, shape, raw bytes)."""
    header, off, blobs = {}, 0, []
    for name, (dt, shape, data) in tensors.items():
        data = bytes(data)
        header[name] = {"dtype": dt, "shape": list(shape), "data_offsets": [off, off + len(data)]}
        blobs.append(data)
        off += len(data)
    h = json.dumps(header).encode()
    h += b" " * ((-len(h)) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))


def bf16_bytes(x: np.ndarray) -> bytes:
    u = np.asarray(x, dtype=np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16).tobytes()
