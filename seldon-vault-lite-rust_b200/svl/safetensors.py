"""Strict Safetensors reader (reference src/binary/safetensors.rs:69-123).

Layout: an 8-byte little-endian header length, a JSON header mapping tensor
names to {dtype, shape, data_offsets}, then the raw tensor bytes.  Only F32
and BF16 are accepted (the reference decodes nothing else); offsets must be in
bounds, ordered and consistent with the shape.  BF16 is widened to FP32 with
the exact bit shift of src/binary/bf16.rs:40 when ``to_f32`` is requested.
"""

from __future__ import annotations

import json
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

from . import errors

MAX_HEADER_BYTES = 100 * 1024 * 1024
_DTYPES = {"F32": (np.float32, 4), "BF16": (np.uint16, 2)}


@dataclass
class TensorEntry:
    name: str
    dtype: str  # "F32" | "BF16"
    shape: tuple[int, ...]
    raw: np.ndarray  # float32 or uint16 (BF16 bits), flat

    def to_f32(self) -> np.ndarray:
        if self.dtype == "F32":
            return self.raw.reshape(self.shape)
        bits = self.raw.astype(np.uint32) << 16
        return bits.view(np.float32).reshape(self.shape)


def parse(data: bytes | memoryview) -> dict[str, TensorEntry]:
    buf = memoryview(data)
    if len(buf) < 8:
        raise errors.CorruptError("Safetensors file is shorter than its header length")
    (hlen,) = struct.unpack("<Q", buf[:8])
    if hlen > MAX_HEADER_BYTES or 8 + hlen > len(buf):
        raise errors.CorruptError("Safetensors header length is out of bounds")
    try:
        header = json.loads(bytes(buf[8 : 8 + hlen]).decode("utf-8"))
    except (UnicodeDecodeError, json.JSONDecodeError):
        raise errors.CorruptError("Safetensors header is not valid JSON") from None
    body = buf[8 + hlen :]
    out: dict[str, TensorEntry] = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dtype = meta.get("dtype")
        if dtype not in _DTYPES:
            raise errors.UnsupportedError(f"tensor {name} has unsupported dtype {dtype}")
        shape = tuple(int(s) for s in meta["shape"])
        begin, end = (int(x) for x in meta["data_offsets"])
        np_dtype, size = _DTYPES[dtype]
        numel = int(np.prod(shape)) if shape else 1
        if begin > end or end > len(body) or end - begin != numel * size:
            raise errors.CorruptError(f"tensor {name} has inconsistent data offsets")
        raw = np.frombuffer(body[begin:end], dtype=np_dtype)
        out[name] = TensorEntry(name, dtype, shape, raw)
    return out


def load(path: str | Path) -> dict[str, TensorEntry]:
    return parse(Path(path).read_bytes())


def write(path: str | Path, tensors: dict[str, np.ndarray]) -> None:
    """Writes F32 tensors in the same container format (test fixtures)."""
    header = {}
    offset = 0
    blobs = []
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr, dtype=np.float32)
        header[name] = {"dtype": "F32", "shape": list(arr.shape), "data_offsets": [offset, offset + arr.nbytes]}
        offset += arr.nbytes
        blobs.append(arr.tobytes())
    hjson = json.dumps(header, separators=(",", ":")).encode()
    hjson += b" " * ((8 - len(hjson) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hjson)))
        f.write(hjson)
        for b in blobs:
            f.write(b)
