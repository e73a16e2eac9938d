"""The reference's .bin model format (src/loader.js:5-77) on the host core.

    magic "JSTORCH\\0" (8 bytes) | version u32 LE | tensor count u32 LE |
    header size u64 LE | header JSON (utf-8) | float32 data, concatenated

header = {"tensors": {key: {"shape": [...], "dtype": "float32", "offset": bytes,
"size": elements}}, "config": {...}}; offsets are relative to the data start.

load_model maps the file and uploads the whole data region with ONE staged
copy (jst_copy_h2d: pinned, double-buffered), then hands out each tensor as a
view of that device block -- the reference instead issues one synchronous
pageable cudaMemcpy per tensor (loader.js:41 -> Tensor.fromBuffer).  The
views keep the block alive.  save_model writes byte-for-byte what
saveModel (loader.js:46-77) writes: the same field order, JSON without
spaces, version 1.
"""
from __future__ import annotations

import json
import mmap
import struct

import numpy as np

MAGIC = b"JSTORCH\0"


def _core():
    from . import _core as c
    return c


def read_header(buf) -> tuple[int, int, dict, int]:
    """(version, tensor count, header dict, data offset) of a .bin image, with
    the checks loadModel makes (loader.js:21-32) plus bounds checks."""
    if len(buf) < 24 or bytes(buf[:8]) != MAGIC:
        raise ValueError(f'Invalid .bin file: bad magic "{bytes(buf[:8])!r}"')
    version, count, hsize = struct.unpack_from("<IIQ", buf, 8)
    if 24 + hsize > len(buf):
        raise ValueError("Invalid .bin file: header runs past the end of the file")
    header = json.loads(bytes(buf[24:24 + hsize]).decode("utf-8"))
    return version, count, header, 24 + hsize


def load_model(path: str):
    """loadModel (loader.js:18-44): returns (state_dict of _core.Tensor, config)."""
    core = _core()
    with open(path, "rb") as f:
        size = f.seek(0, 2)
        if size == 0:
            raise ValueError("Invalid .bin file: empty")
        with mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as mm:
            _, _, header, data0 = read_header(mm)
            tensors = header.get("tensors", {})
            end = 0
            for key, info in tensors.items():
                off, n = int(info["offset"]), int(info["size"])
                if off % 4 or off < 0 or n < 0 or data0 + off + 4 * n > size:
                    raise ValueError(f"Invalid .bin file: tensor {key!r} lies outside the data region")
                if int(np.prod(info["shape"], dtype=np.int64)) != n:
                    raise ValueError(f"Invalid .bin file: tensor {key!r} shape does not match its size")
                end = max(end, off + 4 * n)
            state = {}
            if end:
                data = np.frombuffer(mm, dtype=np.float32, count=end // 4, offset=data0)
                block = core.Tensor.fromBuffer(data, [end // 4])  # one staged upload
                del data
                for key, info in tensors.items():
                    off, n = int(info["offset"]) // 4, int(info["size"])
                    shape = [int(d) for d in info["shape"]]
                    state[key] = block.slice(0, off, off + n).reshape(shape) if n else \
                        core.Tensor.fromBuffer(np.zeros(0, np.float32), shape)
            else:
                for key, info in tensors.items():
                    state[key] = core.Tensor.fromBuffer(np.zeros(0, np.float32), [int(d) for d in info["shape"]])
    return state, header.get("config") or {}


def save_model(path: str, state_dict: dict, config: dict | None = None) -> None:
    """saveModel (loader.js:46-77): tensors (anything with toArray() or a numpy
    array) in insertion order."""
    tensors, blobs, offset = {}, [], 0
    for key, t in state_dict.items():
        arr = np.ascontiguousarray(t.toArray() if hasattr(t, "toArray") else t, dtype=np.float32)
        tensors[key] = {"shape": [int(d) for d in arr.shape], "dtype": "float32", "offset": offset,
                        "size": int(arr.size)}
        blobs.append(arr.tobytes())
        offset += arr.size * 4
    header = json.dumps({"tensors": tensors, "config": config or {}}, separators=(",", ":"),
                        ensure_ascii=False).encode("utf-8")
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<IIQ", 1, len(tensors), len(header)))
        f.write(header)
        for b in blobs:
            f.write(b)
