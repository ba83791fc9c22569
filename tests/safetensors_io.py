"""Test helper: write safetensors files and model directories (the format
`safetensors 0.4.5` reads, Cargo.lock:2049-2051): 8-byte little-endian header length,
a JSON header {name: {dtype, shape, data_offsets}}, then the raw little-endian bytes."""
import json
import struct
from pathlib import Path

import numpy as np

_DTYPES = {np.dtype(np.float16): "F16", np.dtype(np.float32): "F32", np.dtype(np.int8): "I8",
           np.dtype(np.uint8): "U8", np.dtype(np.int32): "I32", np.dtype(np.int64): "I64",
           np.dtype(np.float64): "F64"}


def bf16(a: np.ndarray) -> tuple:
    """f32 values -> ("BF16", uint16 bits) by round-to-nearest-even (how bf16 checkpoints
    are produced); the loader then narrows bf16 -> f16."""
    x = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = ((x >> 16) & 1) + 0x7FFF
    return "BF16", ((x + r) >> 16).astype(np.uint16)


def write_safetensors(path, tensors: dict, metadata: dict | None = None):
    """tensors: name -> ndarray, or (dtype string, ndarray of the element bytes)."""
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, v in tensors.items():
        dt, arr = v if isinstance(v, tuple) else (_DTYPES[np.asarray(v).dtype], v)
        arr = np.ascontiguousarray(arr)
        b = arr.tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def write_model_dir(d, shards: list, config: dict | None = None):
    """shards: list of tensor dicts; more than one -> model-0000k-of-0000n.safetensors +
    model.safetensors.index.json."""
    d = Path(d)
    d.mkdir(parents=True, exist_ok=True)
    if len(shards) == 1:
        write_safetensors(d / "model.safetensors", shards[0])
    else:
        wm = {}
        for k, t in enumerate(shards):
            fn = f"model-{k + 1:05d}-of-{len(shards):05d}.safetensors"
            write_safetensors(d / fn, t)
            wm.update({name: fn for name in t})
        (d / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": wm}))
    if config is not None:
        (d / "config.json").write_text(json.dumps(config))
    return d
