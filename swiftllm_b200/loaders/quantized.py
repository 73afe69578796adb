"""GPTQ / AWQ checkpoints: the tensor getter the weight loader sees.

A quantised HF checkpoint stores ``<prefix>.qweight``, ``.qzeros``,
``.scales`` (and GPTQ's ``.g_idx``) instead of ``<prefix>.weight``, and names
the method in config.json's ``quantization_config``. ``wrap_quantized``
returns a getter that answers ``<prefix>.weight`` with the dequantised
fp32 matrix, so the per-rank slicing and the QKV / gate-up fusion of the
regular loader apply unchanged; the model then re-packs each (sharded,
fused) projection into the int4 tile layout with the checkpoint's group
size (ops.int4.quantize). Where a group's codes span 0..15 - the usual
case for GPTQ / AWQ - the re-packed codes, scales and zero points equal
the checkpoint's up to the bf16 rounding of the scale.

Parity: crates/swiftllm-core/src/config.rs:184-215 (QuantizationConfig with
GPTQ / AWQ methods and group size; the reference has no loader for them).
"""

from __future__ import annotations

import json
import os
from typing import Callable, Optional, Tuple

import torch

from ..ops import int4


def quant_config(model_dir: str) -> Optional[dict]:
    """config.json's quantization_config (or quantize_config.json), or None."""
    if not os.path.isdir(model_dir):
        return None
    for name, key in (("config.json", "quantization_config"), ("quantize_config.json", None)):
        p = os.path.join(model_dir, name)
        if os.path.exists(p):
            with open(p) as f:
                d = json.load(f)
            d = d.get(key) if key else d
            if d:
                return d
    return None


def wrap_quantized(get: Callable[[str], Optional[torch.Tensor]], model_dir: str
                   ) -> Tuple[Callable[[str], Optional[torch.Tensor]], Optional[Tuple[str, int]]]:
    """(getter, (method, group) or None). Without a GPTQ / AWQ config the
    getter is returned unchanged."""
    qc = quant_config(model_dir)
    method = (qc or {}).get("quant_method", (qc or {}).get("method"))
    if method is None and qc is not None and "bits" in qc:
        method = "gptq"  # AutoGPTQ's quantize_config.json has no method field
    if method not in ("gptq", "awq"):
        return get, None
    bits = int(qc.get("bits", qc.get("w_bit", 4)))
    if bits != 4:
        raise NotImplementedError(f"{method} with {bits}-bit weights is not supported (4-bit is)")
    group = int(qc.get("group_size", qc.get("q_group_size", 128)))
    if qc.get("desc_act"):
        raise NotImplementedError("GPTQ act-order (desc_act) checkpoints are not supported")
    version = str(qc.get("version", "")).lower()
    if method == "awq" and version not in ("", "gemm"):
        raise NotImplementedError(f"AWQ version {version!r} is not supported (GEMM packing is)")

    def qget(name: str) -> Optional[torch.Tensor]:
        t = get(name)
        if t is not None or not name.endswith(".weight"):
            return t
        pre = name[: -len(".weight")]
        qw = get(pre + ".qweight")
        if qw is None:
            return None
        qz, sc = get(pre + ".qzeros"), get(pre + ".scales")
        if method == "gptq":
            q, z, s, g = int4.from_gptq(qw, qz, sc, get(pre + ".g_idx"),
                                        group=group if group > 0 else None)
        else:
            q, z, s, g = int4.from_awq(qw, qz, sc, group=group if group > 0 else None)
        return int4.dequantize_codes(q, z, s, g)

    return qget, (method, group if group > 0 else 0)
