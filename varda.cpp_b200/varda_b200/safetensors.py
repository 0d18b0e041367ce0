"""Plain safetensors read/write with numpy, in the layout varda.cpp's model files use.

Layout (the reference's format contract, src/varda/format.h:1-85): u64 little-endian header length
N, N bytes of JSON (space padded so 8 + N is a multiple of 8), then the packed tensor data.
Tensors are written widest element type first so every tensor starts at a multiple of its element
size, which the engine's loader requires (format.cpp:123 in the reference).
"""
from __future__ import annotations

import json
import os
import struct

import numpy as np

DTYPES = {np.dtype(np.float32): "F32", np.dtype(np.float16): "F16", np.dtype(np.float64): "F64",
          np.dtype(np.int64): "I64", np.dtype(np.int32): "I32", np.dtype(np.uint8): "U8",
          np.dtype(np.int8): "I8", np.dtype(np.int16): "I16"}
NP = {v: k for k, v in DTYPES.items()}


def write(path: str, tensors: dict, metadata: dict) -> None:
    """Writes atomically (temporary name in the same directory, then rename)."""
    hdr = {"__metadata__": {k: str(v) for k, v in metadata.items()}}
    order = sorted(tensors.items(), key=lambda kv: -np.asarray(kv[1]).dtype.itemsize)
    off = 0
    arrs = []
    for name, a in order:
        a = np.ascontiguousarray(a)
        if a.dtype.byteorder == ">":
            a = a.astype(a.dtype.newbyteorder("<"))
        nb = a.nbytes
        hdr[name] = {"dtype": DTYPES[a.dtype], "shape": list(a.shape), "data_offsets": [off, off + nb]}
        off += nb
        arrs.append(a)
    h = json.dumps(hdr).encode()
    h += b" " * ((8 - (8 + len(h)) % 8) % 8)
    tmp = f"{path}.tmp.{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for a in arrs:
            f.write(memoryview(a.reshape(-1).view(np.uint8)))
    os.replace(tmp, path)


def read(path: str):
    """Returns ({name: ndarray view of a read-only map}, metadata)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        hdr = json.loads(f.read(n))
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for k, v in hdr.items():
        if k == "__metadata__":
            continue
        a, b = v["data_offsets"]
        dt = NP[v["dtype"]]
        out[k] = np.frombuffer(mm, dtype=dt, count=(b - a) // dt.itemsize, offset=8 + n + a).reshape(v["shape"])
    return out, hdr.get("__metadata__", {})
