"""Minimal safetensors container I/O with numpy, for writing and reading the synthetic checkpoints.

Format: 8-byte little-endian header length, a JSON header mapping tensor names to
{dtype, shape, data_offsets}, then the raw little-endian tensor bytes. The engine's C++ loader reads
the same container (the reference mmaps it in src/laya.cpp:53-71).
"""
import json
import struct

import numpy as np

_DT = {"F32": np.float32, "F16": np.float16, "I32": np.int32, "I64": np.int64, "BF16": np.uint16}
_NAME = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.int32): "I32",
         np.dtype(np.int64): "I64"}


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bits (finite inputs)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    r = ((u >> 16) & 1) + 0x7FFF
    return ((u + r) >> 16).astype(np.uint16)


def write(path, tensors, bf16_names=()):
    """tensors: ordered mapping name -> np.ndarray. Names in bf16_names are stored as BF16."""
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        if name in bf16_names:
            raw = f32_to_bf16(arr).tobytes()
            dt = "BF16"
        else:
            arr = np.ascontiguousarray(arr)
            raw = arr.tobytes()
            dt = _NAME[arr.dtype]
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def read(path, as_f32=True):
    """Returns an ordered dict name -> np.ndarray (floating tensors as fp32 when as_f32)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        base = 8 + n
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        a, b = meta["data_offsets"]
        arr = np.frombuffer(mm[base + a:base + b], dtype=_DT[meta["dtype"]]).reshape(meta["shape"])
        if meta["dtype"] == "BF16":
            arr = bf16_to_f32(arr) if as_f32 else arr
        elif as_f32 and meta["dtype"] == "F16":
            arr = arr.astype(np.float32)
        out[name] = np.array(arr)
    return out
