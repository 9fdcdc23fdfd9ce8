"""Writes safetensors files for the checkpoint-loader tests (test infrastructure, not product code).

Format (as SafeTensors.swift:19-45 reads it): u64 little-endian header length, a JSON header
{name: {"dtype", "shape", "data_offsets": [begin, end]}} (offsets relative to the data section)
with an optional "__metadata__" entry, then the tensor bytes.
"""
from __future__ import annotations

import json
import struct

import numpy as np

DTYPE_BYTES = {"BF16": 2, "F32": 4, "F16": 2, "I64": 8}


def encode(tensors: dict, metadata: dict | None = None) -> bytes:
    """tensors: name -> (dtype, shape, raw bytes). Returns the whole file."""
    header = {}
    if metadata is not None:
        header["__metadata__"] = metadata
    data = bytearray()
    for name, (dtype, shape, raw) in tensors.items():
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [len(data), len(data) + len(raw)]}
        data += raw
    head = json.dumps(header).encode()
    head += b" " * (-len(head) % 8)  # the format pads the header to 8 bytes
    return struct.pack("<Q", len(head)) + head + bytes(data)


def write(path, tensors: dict, metadata: dict | None = None) -> None:
    with open(path, "wb") as f:
        f.write(encode(tensors, metadata))


def bf16_bits(rng: np.random.Generator, n: int) -> np.ndarray:
    """Random finite bf16 bit patterns (values ~ N(0, 0.5))."""
    x = (rng.standard_normal(n) * 0.5).astype(np.float32)
    return (x.view(np.uint32) >> 16).astype(np.uint16)
