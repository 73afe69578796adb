"""Checkpoint opening: format detection and a name -> tensor getter.

Parity: crates/swiftllm-models/src/loaders/mod.rs (detect_format :51-81),
huggingface.rs (shard discovery via model.safetensors.index.json :276-327),
safetensors.rs and gguf.rs (parsers; the C++ versions live in
csrc/core/loaders.cpp).
"""

from __future__ import annotations

import glob
import json
import os
from typing import Dict, Optional

import numpy as np
import torch

from .. import _core

_ST_DTYPES = {
    "F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16, "F64": torch.float64,
    "I8": torch.int8, "U8": torch.uint8, "I16": torch.int16, "I32": torch.int32, "I64": torch.int64,
    "F8_E4M3": torch.float8_e4m3fn, "F8_E5M2": torch.float8_e5m2, "BOOL": torch.bool,
}


def detect_format(path: str) -> str:
    if os.path.isdir(path):
        if glob.glob(os.path.join(path, "*.safetensors")):
            return "safetensors"
        if glob.glob(os.path.join(path, "*.gguf")):
            return "gguf"
        if glob.glob(os.path.join(path, "*.bin")) or glob.glob(os.path.join(path, "*.pt")):
            return "pt"
        raise ValueError(f"no weights found in {path}")
    low = path.lower()
    for ext, fmt in ((".safetensors", "safetensors"), (".gguf", "gguf"), (".ggml", "gguf"),
                     (".bin", "pt"), (".pt", "pt"), (".pth", "pt")):
        if low.endswith(ext):
            return fmt
    raise ValueError(f"unknown checkpoint format: {path}")


class SafeTensorsCheckpoint:
    """All shards of a safetensors checkpoint; tensors are zero-copy views of
    the mapped files until sliced and copied to the device."""

    def __init__(self, path: str):
        files = [path] if os.path.isfile(path) else sorted(glob.glob(os.path.join(path, "*.safetensors")))
        index = os.path.join(path, "model.safetensors.index.json") if os.path.isdir(path) else None
        if index and os.path.exists(index):
            with open(index) as f:
                wm = json.load(f)["weight_map"]
            files = sorted({os.path.join(path, v) for v in wm.values()})
        self.files = [_core.SafeTensorsFile(f) for f in files]
        self.where: Dict[str, _core.SafeTensorsFile] = {}
        for f in self.files:
            for k in f.keys():
                self.where[k] = f

    def keys(self):
        return list(self.where)

    def get(self, name: str) -> Optional[torch.Tensor]:
        f = self.where.get(name)
        if f is None:
            return None
        dt = _ST_DTYPES[f.dtype(name)]
        raw = f.raw(name)
        t = torch.from_numpy(np.asarray(raw)).view(dt)
        return t.view(f.shape(name))


class TorchCheckpoint:
    def __init__(self, path: str):
        files = [path] if os.path.isfile(path) else sorted(
            glob.glob(os.path.join(path, "*.bin")) + glob.glob(os.path.join(path, "*.pt")))
        self.sd = {}
        for f in files:
            self.sd.update(torch.load(f, map_location="cpu", weights_only=True))

    def keys(self):
        return list(self.sd)

    def get(self, name):
        return self.sd.get(name)


def open_checkpoint(path: str, fmt: str = "auto"):
    if fmt in ("auto",):
        fmt = detect_format(path)
    if fmt == "safetensors":
        return SafeTensorsCheckpoint(path)
    if fmt == "gguf":
        from .gguf import GgufCheckpoint
        if os.path.isdir(path):
            path = sorted(glob.glob(os.path.join(path, "*.gguf")))[0]
        return GgufCheckpoint(path)
    if fmt == "pt":
        return TorchCheckpoint(path)
    raise ValueError(fmt)
