"""Checkpoint conversion: GGUF / safetensors / .bin in, a single safetensors
file with HF tensor names out. Also the safetensors writer used by tests.

The safetensors layout (8-byte little-endian header length, JSON header of
{name: {dtype, shape, data_offsets}}, raw little-endian data) is the public
format; the parser lives in csrc/core/loaders.cpp.
"""

from __future__ import annotations

import json
import struct
from typing import Dict

import numpy as np
import torch

_DT = {torch.float32: "F32", torch.float16: "F16", torch.bfloat16: "BF16", torch.int8: "I8",
       torch.int32: "I32", torch.int64: "I64", torch.uint8: "U8"}


def save_safetensors(tensors: Dict[str, torch.Tensor], path: str,
                     metadata: Dict[str, str] = None) -> None:
    header = {}
    off = 0
    blobs = []
    for name, t in tensors.items():
        t = t.detach().contiguous().cpu()
        raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _DT[t.dtype], "shape": list(t.shape),
                        "data_offsets": [off, off + len(raw)]}
        off += len(raw)
        blobs.append(raw)
    if metadata:
        header["__metadata__"] = metadata
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def convert(src: str, dst: str, dtype: str = "bfloat16") -> int:
    from . import open_checkpoint
    dt = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}[dtype]
    ck = open_checkpoint(src)
    out = {}
    for k in ck.keys():
        if ".experts_packed." in k:
            # GGUF packs experts; emit HF per-expert names
            i, w = k.split(".")[2], k.split(".")[-1]
            packed = ck.get(k)
            for e in range(packed.shape[0]):
                out[f"model.layers.{i}.block_sparse_moe.experts.{e}.{w}.weight"] = packed[e].to(dt)
            continue
        t = ck.get(k)
        out[k] = t.to(dt) if t.is_floating_point() else t
    save_safetensors(out, dst, {"format": "pt", "converted_by": "swiftllm_b200"})
    return len(out)
