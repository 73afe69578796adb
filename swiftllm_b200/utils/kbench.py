"""Kernel micro-benchmarks (CUDA-event timing, L2 flushed between runs) and
single-shot runners used for ncu captures.

  python -m swiftllm_b200.utils.kbench gemm --shape 256,12288,4096 [--once]
  python -m swiftllm_b200.utils.kbench decode --shape 256,900,32,32 [--splits 1] [--once]
  python -m swiftllm_b200.utils.kbench prefill --shape 8,1024,32,8
  python -m swiftllm_b200.utils.kbench sweep [--json out.json]

Timing rule: 3 warm-up runs, then each timed run writes a 256 MB buffer
(larger than the 126 MB L2) before it, is bracketed by CUDA events on the
current stream with synchronisation on both sides; the median is reported.
Bandwidth / FLOP rates are also given as fractions of MEASURED_PEAKS.json.
``--once`` runs the op four times without timing (for ncu -s 2 -c 1).
"""

from __future__ import annotations

import argparse
import json
import math
import sys

import torch

from ..ops import cuda_ext
from .timing import measured_peaks


def _time(fn, iters=20):
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(3):
        fn()
    ts = []
    for _ in range(iters):
        flush.zero_()
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        torch.cuda.synchronize()
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    ts.sort()
    return ts[len(ts) // 2]


def gemm_case(T, N, K, once=False, cublas=True):
    C = cuda_ext()
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    y = torch.empty(T, N, device="cuda", dtype=torch.bfloat16)
    if once:
        for _ in range(4):
            C.gemm(y, x, w, None)
        torch.cuda.synchronize()
        return {}
    pk = measured_peaks()
    ms = _time(lambda: C.gemm(y, x, w, None))
    byts = (N * K + T * K + T * N) * 2
    fl = 2.0 * T * N * K
    r = {"op": "gemm", "T": T, "N": N, "K": K, "plan": C.gemm_plan(N, T, K), "ms": round(ms, 4),
         "TB/s": round(byts / ms / 1e9, 2), "TFLOP/s": round(fl / ms / 1e9, 1),
         "frac_bw": round(byts / ms / 1e9 / (pk["hbm_gbs"] / 1e3), 3),
         "frac_flops": round(fl / ms / 1e9 / pk["bf16_tflops"], 3)}
    if cublas:
        r["cublas_ms"] = round(_time(lambda: torch.matmul(x, w.t())), 4)
    return r


def _pool(S, ctx, Hq, Hkv, D=128, bs=16, L=1):
    nbp = (ctx + bs - 1) // bs
    kv = torch.randn(S * nbp, L, 2, Hkv, bs, D, device="cuda").bfloat16()
    bt = torch.randperm(S * nbp, device="cuda").int().view(S, nbp)
    return kv, bt


def decode_case(S, ctx, Hq, Hkv, splits=1, once=False, D=128):
    C = cuda_ext()
    kv, bt = _pool(S, ctx, Hq, Hkv, D)
    q = torch.randn(S, Hq, D, device="cuda").bfloat16()
    sl = torch.full((S,), ctx, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    ws = torch.empty(max(1, S * Hq * splits * (D + 2)), device="cuda")
    fn = lambda: C.paged_decode(out, q, kv, 0, bt, sl, S, splits, 1 / math.sqrt(D), 0, ws)  # noqa: E731
    if once:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        return {}
    ms = _time(fn)
    byts = S * ctx * Hkv * D * 2 * 2
    pk = measured_peaks()
    return {"op": "paged_decode", "S": S, "ctx": ctx, "Hq": Hq, "Hkv": Hkv, "splits": splits,
            "ms": round(ms, 4), "TB/s": round(byts / ms / 1e9, 2),
            "frac_bw": round(byts / ms / 1e9 / (pk["hbm_gbs"] / 1e3), 3)}


def prefill_case(S, L, Hq, Hkv, once=False, D=128):
    C = cuda_ext()
    kv, bt = _pool(S, L, Hq, Hkv, D)
    q = torch.randn(S * L, Hq, D, device="cuda").bfloat16()
    qs = torch.arange(0, S * L + 1, L, dtype=torch.int32, device="cuda")
    sl = torch.full((S,), L, dtype=torch.int32, device="cuda")
    out = torch.empty_like(q)
    fn = lambda: C.paged_prefill(out, q, kv, 0, bt, qs, sl, 0, S, L, 1 / math.sqrt(D), 0)  # noqa: E731
    if once:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        return {}
    ms = _time(fn)
    fl = 4.0 * S * Hq * D * L * L / 2  # causal
    pk = measured_peaks()
    return {"op": "paged_prefill", "S": S, "L": L, "Hq": Hq, "Hkv": Hkv, "ms": round(ms, 4),
            "TFLOP/s": round(fl / ms / 1e9, 1), "frac_flops": round(fl / ms / 1e9 / pk["bf16_tflops"], 3)}


def sweep():
    res = []
    for T, N, K in [(256, 12288, 4096), (256, 4096, 4096), (256, 22016, 4096), (256, 4096, 11008),
                    (256, 32000, 4096), (8192, 12288, 4096), (8192, 22016, 4096),
                    (8192, 4096, 11008)]:
        res.append(gemm_case(T, N, K))
        print(json.dumps(res[-1]), flush=True)
    for S, ctx, Hq, Hkv in [(256, 900, 32, 32), (256, 900, 32, 8), (64, 2000, 32, 32)]:
        res.append(decode_case(S, ctx, Hq, Hkv))
        print(json.dumps(res[-1]), flush=True)
    for S, L, Hq, Hkv in [(8, 1024, 32, 32), (2, 4096, 32, 8)]:
        res.append(prefill_case(S, L, Hq, Hkv))
        print(json.dumps(res[-1]), flush=True)
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("op", choices=["gemm", "decode", "prefill", "sweep"])
    ap.add_argument("--shape", default=None)
    ap.add_argument("--splits", type=int, default=1)
    ap.add_argument("--once", action="store_true")
    ap.add_argument("--json", default=None)
    a = ap.parse_args(argv)
    if a.op == "sweep":
        res = sweep()
    else:
        shp = [int(v) for v in a.shape.split(",")]
        if a.op == "gemm":
            res = gemm_case(*shp, once=a.once)
        elif a.op == "decode":
            res = decode_case(*shp, splits=a.splits, once=a.once)
        else:
            res = prefill_case(*shp, once=a.once)
        print(json.dumps(res) if res else "ok")
    if a.json:
        with open(a.json, "w") as f:
            json.dump(res, f, indent=1)


if __name__ == "__main__":
    sys.exit(main())
