"""Writes and reads safetensors files (8-byte little-endian header length, JSON header, raw little-endian data) for
the LoRA and checkpoint tests; the format as the safetensors project documents it, written here so no extra package
is needed."""
import json
import struct

import numpy as np
import torch


def write(path, tensors, metadata=None, dtype="BF16"):
    """tensors: {name: array-like}; stored as BF16 (round to nearest even) or F32; dtype one of those or a
    {name: dtype} map."""
    header, blobs, off = {}, [], 0
    for name, a in tensors.items():
        t = torch.as_tensor(np.asarray(a, np.float32))
        dt = dtype[name] if isinstance(dtype, dict) else dtype
        if dt == "BF16":
            raw = t.bfloat16().view(torch.int16).numpy().tobytes()
        else:
            raw = t.numpy().astype("<f4").tobytes()
        header[name] = {"dtype": dt, "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
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


def read(path):
    """({name: float32 array}, {name: dtype}, metadata) of a file of BF16 and F32 tensors."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        data = f.read()
    meta = header.pop("__metadata__", {})
    tensors, dtypes = {}, {}
    for name, info in header.items():
        a, b = info["data_offsets"]
        raw = data[a:b]
        if info["dtype"] == "BF16":
            v = (np.frombuffer(raw, "<u2").astype(np.uint32) << 16).view(np.float32)
        else:
            v = np.frombuffer(raw, "<f4")
        tensors[name] = v.reshape(info["shape"]).copy()
        dtypes[name] = info["dtype"]
    return tensors, dtypes, meta


def bf16_values(a):
    """The values a BF16 file stores for `a`, as float32."""
    return torch.as_tensor(np.asarray(a, np.float32)).bfloat16().float()
