"""Writes small GGUF v3 files for the tests (the published ggml GGUF layout): tensors as F32,
F16 or Q8_0 (blocks of an f16 scale d and 32 int8 q, W = q * d). Test infrastructure only."""
from __future__ import annotations

import struct

import numpy as np

ALIGN = 32
TYPES = {"f32": 0, "f16": 1, "q8_0": 8}


def _str(s: str) -> bytes:
    b = s.encode()
    return struct.pack("<Q", len(b)) + b


def q8_0_blocks(q: np.ndarray, d: np.ndarray) -> np.ndarray:
    """int8 q [N][K] and scales d [N][K/32] (f16-representable) -> the q8_0 bytes [N][K/32 * 34]."""
    n, k = q.shape
    blocks = np.zeros((n, k // 32, 34), np.uint8)
    blocks[:, :, :2] = d.astype(np.float16).view(np.uint8).reshape(n, k // 32, 2)
    blocks[:, :, 2:] = q.astype(np.int8).view(np.uint8).reshape(n, k // 32, 32)
    return blocks.reshape(n, -1)


def write(path: str, tensors: list, *, version: int = 3, alignment: int = ALIGN):
    """tensors: (name, kind, array) with kind "f32" / "f16" (array of that shape, row-major)
    or "q8_0" (array = (q int8 [N][K], d [N][K/32]))."""
    infos, blobs, offset = [], [], 0
    for name, kind, arr in tensors:
        if kind == "q8_0":
            q, d = arr
            data = q8_0_blocks(q, d).tobytes()
            shape = q.shape
        else:
            a = np.ascontiguousarray(arr, dtype=np.float32 if kind == "f32" else np.float16)
            data, shape = a.tobytes(), a.shape
        dims = list(reversed(shape))  # innermost first
        infos.append(_str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", x) for x in dims)
                     + struct.pack("<IQ", TYPES[kind], offset))
        pad = (-len(data)) % alignment
        blobs.append(data + b"\0" * pad)
        offset += len(data) + pad
    meta = [_str("general.architecture") + struct.pack("<I", 8) + _str("ptts-test"),
            _str("general.alignment") + struct.pack("<II", 4, alignment)]
    head = b"GGUF" + struct.pack("<IQQ", version, len(tensors), len(meta)) + b"".join(meta) + b"".join(infos)
    head += b"\0" * ((-len(head)) % alignment)
    with open(path, "wb") as f:
        f.write(head)
        for b in blobs:
            f.write(b)
