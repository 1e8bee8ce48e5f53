"""Minimal safetensors reader/writer over numpy (no torch, no safetensors package).

The format (8-byte little-endian header length, a JSON header mapping tensor
names to dtype/shape/data_offsets, then the raw little-endian bytes) is what
MLX's ``mx.save_safetensors`` writes for mlx-lm converted checkpoints; the
reference engine reads every ``*.safetensors`` file in the artifact directory
(native/hyperion_mlx/src/weights_loader.cc:72-154). BF16 tensors are returned as
``uint16`` bit patterns, U32 packed weights as ``uint32``.
"""
from __future__ import annotations

import json
import os
import struct
from typing import Dict

import numpy as np

_DT_TO_NP = {
    "BF16": np.uint16,
    "F16": np.float16,
    "F32": np.float32,
    "U32": np.uint32,
    "I32": np.int32,
    "U8": np.uint8,
}
_NP_TO_DT = {
    np.dtype(np.uint16): "BF16",
    np.dtype(np.float16): "F16",
    np.dtype(np.float32): "F32",
    np.dtype(np.uint32): "U32",
    np.dtype(np.int32): "I32",
    np.dtype(np.uint8): "U8",
}


def read_safetensors(path: str) -> Dict[str, np.ndarray]:
    """Read one file; returns name -> array (BF16 as uint16 bit patterns)."""
    with open(path, "rb") as f:
        (hlen,) = struct.unpack("<Q", f.read(8))
        header = json.loads(f.read(hlen))
        base = 8 + hlen
        data = np.memmap(path, dtype=np.uint8, mode="r")
    out = {}
    for name, meta in header.items():
        if name == "__metadata__":
            continue
        dt = _DT_TO_NP[meta["dtype"]]
        lo, hi = meta["data_offsets"]
        arr = np.frombuffer(data[base + lo: base + hi], dtype=dt)
        out[name] = arr.reshape(meta["shape"])
    return out


def read_checkpoint_dir(path: str) -> Dict[str, np.ndarray]:
    """Merge every ``*.safetensors`` file in ``path`` (sorted), like the reference loader."""
    files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors shards found in {path}")
    merged: Dict[str, np.ndarray] = {}
    for fn in files:
        merged.update(read_safetensors(os.path.join(path, fn)))
    return merged


def write_safetensors(path: str, tensors: Dict[str, np.ndarray]) -> None:
    """Write tensors (uint16 arrays are tagged BF16)."""
    header = {}
    offset = 0
    order = sorted(tensors)
    for name in order:
        arr = np.ascontiguousarray(tensors[name])
        nbytes = arr.nbytes
        header[name] = {
            "dtype": _NP_TO_DT[arr.dtype],
            "shape": list(arr.shape),
            "data_offsets": [offset, offset + nbytes],
        }
        offset += nbytes
    hbytes = json.dumps(header, separators=(",", ":")).encode()
    pad = (8 - len(hbytes) % 8) % 8
    hbytes += b" " * pad
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hbytes)))
        f.write(hbytes)
        for name in order:
            f.write(np.ascontiguousarray(tensors[name]).tobytes())
