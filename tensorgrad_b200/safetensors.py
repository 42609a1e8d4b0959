"""safetensors container: read (the reference's loader, src/safetensors.ts:49-103)
and write (new: the reference has no writer).

Format: an 8-byte little-endian u64 header length N, an N-byte JSON header, then
one data blob. The header maps each tensor name to {dtype, shape, data_offsets:
[start, end]} (byte offsets into the blob); the reserved "__metadata__" key maps
to free-form string metadata.

Reading is f32-only, as in the reference: integer/bool tensors are bookkeeping
and are skipped and reported, other float dtypes raise rather than being
misread.
"""
from __future__ import annotations

import json
import struct
from typing import Dict, Optional

import numpy as np

INTEGER_DTYPES = {"I64", "I32", "I16", "I8", "U8", "U16", "U32", "U64", "BOOL"}


def loadSafetensors(buf: bytes) -> dict:
    """Returns {"tensors": {name: float32 array}, "shapes": {name: shape},
    "skipped": {name: dtype}, "metadata": {str: str}}."""
    buf = bytes(buf)
    if len(buf) < 8:
        raise ValueError("loadSafetensors: buffer too small to hold the 8-byte header length")
    (hlen,) = struct.unpack_from("<Q", buf, 0)
    hend = 8 + hlen
    if hend > len(buf):
        raise ValueError(f"loadSafetensors: header length {hlen} exceeds buffer ({len(buf)} bytes)")
    try:
        header = json.loads(buf[8:hend].decode("utf-8"))
    except ValueError as e:
        raise ValueError(f"loadSafetensors: header is not valid JSON: {e}") from None
    tensors: Dict[str, np.ndarray] = {}
    shapes: Dict[str, list] = {}
    skipped: Dict[str, str] = {}
    for name, entry in header.items():
        if name == "__metadata__":
            continue
        shapes[name] = list(entry["shape"])
        dtype = entry["dtype"]
        if dtype != "F32":
            if dtype in INTEGER_DTYPES:
                skipped[name] = dtype
                continue
            raise ValueError(f"loadSafetensors: tensor '{name}' has dtype '{dtype}', but tensorgrad is f32-only. "
                             "Convert the checkpoint to f32 offline before loading.")
        start, end = entry["data_offsets"]
        if start > end or hend + end > len(buf):
            raise ValueError(f"loadSafetensors: tensor '{name}' data_offsets [{start}, {end}] out of range")
        numel = int(np.prod(entry["shape"], dtype=np.int64)) if entry["shape"] else 1
        if end - start != numel * 4:
            raise ValueError(f"loadSafetensors: tensor '{name}' byte length {end - start} != {numel} f32 elements * 4 "
                             f"(shape {list(entry['shape'])})")
        tensors[name] = np.frombuffer(buf, np.float32, numel, hend + start).reshape(entry["shape"]).copy()
    return {"tensors": tensors, "shapes": shapes, "skipped": skipped, "metadata": dict(header.get("__metadata__", {}))}


def saveSafetensors(tensors: Dict[str, np.ndarray], metadata: Optional[Dict[str, str]] = None) -> bytes:
    """Serialise f32 tensors (in the given order) and string metadata. The
    header is padded with spaces to a multiple of 8 bytes so every tensor's
    data starts 8-byte aligned in the file."""
    header: Dict[str, dict] = {}
    blobs = []
    off = 0
    for name, arr in tensors.items():
        if name == "__metadata__":
            raise ValueError("saveSafetensors: '__metadata__' is reserved")
        a = np.asarray(arr, dtype=np.float32, order="C")  # keeps 0-d scalars 0-d
        header[name] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    if metadata:
        header["__metadata__"] = {str(k): str(v) for k, v in metadata.items()}
    h = json.dumps(header, separators=(",", ":")).encode("utf-8")
    h += b" " * ((8 - len(h) % 8) % 8)
    return struct.pack("<Q", len(h)) + h + b"".join(blobs)
