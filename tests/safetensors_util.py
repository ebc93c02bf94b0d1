"""Writes safetensors files (8-byte little-endian header length, JSON header, raw little-endian data) for the LoRA
tests; the format as the safetensors project documents it, written here so no extra package is needed."""
import json
import struct

import numpy as np
import torch


def write(path, tensors, metadata=None, dtype="BF16"):
    """tensors: {name: array-like}; stored as BF16 (round to nearest even) or F32."""
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        t = torch.as_tensor(np.asarray(a, np.float32))
        if dtype == "BF16":
            raw = t.bfloat16().view(torch.int16).numpy().tobytes()
        else:
            raw = t.numpy().astype("<f4").tobytes()
        header[name] = {"dtype": dtype, "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def bf16_values(a):
    """The values a BF16 file stores for `a`, as float32."""
    return torch.as_tensor(np.asarray(a, np.float32)).bfloat16().float()
