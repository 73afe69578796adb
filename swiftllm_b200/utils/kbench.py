"""Kernel micro-benchmarks (CUDA-event timing, L2 flushed between runs) and
single-shot runners used for ncu captures.

  python -m swiftllm_b200.utils.kbench gemm --shape 256,12288,4096 [--once]
  python -m swiftllm_b200.utils.kbench decode --shape 256,900,32,32 [--splits 1] [--once]
  python -m swiftllm_b200.utils.kbench prefill --shape 8,1024,32,8
  python -m swiftllm_b200.utils.kbench sweep [--json out.json]
  python -m swiftllm_b200.utils.kbench step --shape 256,700 [--model llama-2-7b] [--eager] [--once]
  python -m swiftllm_b200.utils.kbench w4 [--shape 256x12288x4096,...] [--once]

Timing rule: 3 warm-up runs, then each timed run reads a 256 MB buffer
(larger than the 126 MB L2) before it, is bracketed by CUDA events on the
current stream with synchronisation on both sides; the median is reported.
Bandwidth / FLOP rates are also given as fractions of MEASURED_PEAKS.json.
``--once`` runs the op four times without timing (for ncu -s 2 -c 1).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys

import torch

from ..ops import cuda_ext
from .timing import measured_peaks


def _time(fn, iters=20, flush=True):
    # flush = READ a 256 MB buffer (L2 left full of clean lines). Writing it
    # instead would leave ~126 MB of dirty lines whose write-back lands inside
    # the timed kernel; SWIFT_KBENCH_FLUSH=write selects that variant.
    buf = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    sink = torch.empty((), dtype=torch.float32, device="cuda")
    write = os.environ.get("SWIFT_KBENCH_FLUSH", "read") == "write"
    for _ in range(3):
        fn()
    ts = []
    for _ in range(iters):
        if flush:
            if write:
                buf.zero_()
            else:
                torch.sum(buf, dim=0, out=sink)
        s, e = torch.cuda.Event(True), torch.cuda.Event(True)
        torch.cuda.synchronize()
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ts.append(s.elapsed_time(e))
    ts.sort()
    return ts[len(ts) // 2]


def _time_chain(fns, rounds=5):
    """Back-to-back launches, as in a decode step: ``fns`` (each with its own
    weights, together larger than L2, so every call streams its weight from
    HBM) captured once into a CUDA graph, replayed ``rounds`` times inside
    one event pair; returns ms per call. Host launch cost is excluded, as
    in the engine's graph replays."""
    for f in fns:
        f()
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        with torch.cuda.graph(g, stream=st):
            for f in fns:
                f()
    torch.cuda.current_stream().wait_stream(st)
    g.replay()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(True), torch.cuda.Event(True)
    s.record()
    for _ in range(rounds):
        g.replay()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / (rounds * len(fns))


def gemm_chain_case(T, N, K):
    """Decode-style GEMM timing: many back-to-back calls cycling through
    weight copies totalling > 256 MB; ours (ops.linear dispatch and the 2-SM
    kernel) vs cuBLAS, ms per call."""
    C = cuda_ext()
    x = torch.randn(T, K, device="cuda").bfloat16()
    n_w = max(2, (256 << 20) // (N * K * 2) + 1)
    ws = [(torch.randn(N, K, device="cuda") * 0.02).bfloat16() for _ in range(n_w)]
    y = torch.empty(T, N, device="cuda", dtype=torch.bfloat16)
    t_ours = _time_chain([lambda w=w: C.gemm(y, x, w, None) for w in ws])
    t_g2 = _time_chain([lambda w=w: C.gemm2(y, x, w, None) for w in ws])
    t_dp = _time_chain([lambda w=w: C.gemm2(y, x, w, None, 0) for w in ws])
    t_cb = _time_chain([lambda w=w: torch.matmul(x, w.t(), out=y) for w in ws])
    t_pk = None
    if T <= 256 and N % 128 == 0 and K % 64 == 0:
        # tile-packed weights: every 128 x 64 tile one contiguous 16 KB block
        wps = [w.view(N // 128, 128, K // 64, 64).permute(0, 2, 1, 3).contiguous() for w in ws]
        t_pk = _time_chain([lambda w=w: C.gemm_packed(y, x, w, N, None) for w in wps])
    pk = measured_peaks()
    byts = N * K * 2
    return {"op": "gemm_chain", "T": T, "N": N, "K": K, "ours_us": round(t_ours * 1e3, 1),
            "gemm2_us": round(t_g2 * 1e3, 1), "gemm2_dp_us": round(t_dp * 1e3, 1),
            "cublas_us": round(t_cb * 1e3, 1),
            "packed_1sm_us": round(t_pk * 1e3, 1) if t_pk else None,
            "ours_weight_TB/s": round(byts / t_ours / 1e9, 2),
            "ours_frac_bw": round(byts / t_ours / 1e9 / (pk["hbm_gbs"] / 1e3), 3),
            "plan": C.gemm_plan(N, T, K), "gemm2_plan": C.gemm2_plan(N, T, K)}


def gemm_case(T, N, K, once=False, cublas=True, kernel="gemm", plan=(-1, 0, 0)):
    """kernel: "gemm" (the ops.linear dispatch) or "gemm2" (the 2-SM kernel,
    with an explicit (plan, bn, splits) when plan[0] >= 0)."""
    C = cuda_ext()
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    y = torch.empty(T, N, device="cuda", dtype=torch.bfloat16)
    if once:
        for _ in range(4):
            if kernel == "gemm2":
                C.gemm2(y, x, w, None, *plan)
            else:
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
    r["gemm2_ms"] = round(_time(lambda: C.gemm2(y, x, w, None)), 4)
    r["gemm2_plan"] = C.gemm2_plan(N, T, K)
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
    fn = lambda impl=-1: C.paged_prefill(out, q, kv, 0, bt, qs, sl, 0, S, L, 1 / math.sqrt(D), 0,  # noqa: E731
                                         impl)
    if once:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        return {}
    ms = _time(fn)
    ms_old = _time(lambda: fn(0))
    fl = 4.0 * S * Hq * D * L * L / 2  # causal
    pk = measured_peaks()
    return {"op": "paged_prefill", "S": S, "L": L, "Hq": Hq, "Hkv": Hkv, "ms": round(ms, 4),
            "TFLOP/s": round(fl / ms / 1e9, 1), "frac_flops": round(fl / ms / 1e9 / pk["bf16_tflops"], 3),
            "mma_sync_ms": round(ms_old, 4)}


def step_case(S, ctx, model="llama-2-7b", eager=False, once=False, iters=20):
    """One decode step of the whole model (S sequences at context ctx):
    the engine's ModelRunner with random-init weights, CUDA-graph replay
    unless eager. Reports ms per step and output tokens/s."""
    import numpy as np
    from ..config import EngineConfig
    from ..models.config import load_config
    from ..runtime.model_runner import ModelRunner, StepInput
    mcfg = load_config(model)
    bs = 16
    nbp = (ctx + 1 + bs - 1) // bs
    ec = EngineConfig(model=model, load_format="dummy", dtype="bfloat16", max_model_len=2048,
                      max_num_seqs=max(S, 1), enforce_eager=eager, max_num_batched_tokens=S)
    r = ModelRunner(mcfg, ec, torch.device("cuda", torch.cuda.current_device()), max_model_len=2048)
    r.load_weights()
    r.allocate_kv(S * nbp + 1, 0)
    r.capture_graphs(S)
    tables = np.arange(S * nbp, dtype=np.int32).reshape(S, nbp)
    pos = np.full(S, ctx, dtype=np.int32)
    slots = (tables[:, ctx // bs] * bs + ctx % bs).astype(np.int32)
    ids = np.random.default_rng(0).integers(0, mcfg.vocab_size, S).astype(np.int32)
    ints = np.concatenate([ids, pos, slots, np.arange(S + 1, dtype=np.int32), pos + 1,
                           tables.reshape(-1)]).astype(np.int32)
    e2 = np.zeros((0, 2), np.int64)
    si = StepInput(S, S, S, 1, ctx + 1, nbp, ints, np.arange(S, dtype=np.int32), e2, e2, e2)
    fn = lambda: r.execute(si)  # noqa: E731
    if once:
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        return {}
    for _ in range(3):
        fn()
    ts = []
    for _ in range(iters):
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(True), torch.cuda.Event(True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        ts.append(a.elapsed_time(b))
    ts.sort()
    ms = ts[len(ts) // 2]
    kv = S * (ctx + 1) * mcfg.num_layers * 2 * mcfg.num_kv_heads * mcfg.head_dim * 2
    w = sum(p.numel() for _, p in r.model.named_parameters()) * 2
    pk = measured_peaks()
    return {"op": "decode_step", "model": model, "S": S, "ctx": ctx, "graphs": not eager,
            "ms": round(ms, 3), "tok/s": round(S / ms * 1e3, 1), "weights_GB": round(w / 1e9, 2),
            "kv_GB": round(kv / 1e9, 2), "frac_bw": round((w + kv) / ms / 1e9 / (pk["hbm_gbs"] / 1e3), 3)}


def fp8_case(T, N, K):
    """E4M3 GEMM (per-row scales) vs the bf16 GEMM of the same shape; the fp8
    time includes the activation quantisation kernel."""
    from .. import ops
    C = cuda_ext()
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    fw = ops.fp8_weight(w)
    y = torch.empty(T, N, device="cuda", dtype=torch.bfloat16)
    t8 = _time(lambda: ops.linear(x, fw, out=y))
    t16 = _time(lambda: C.gemm(y, x, w, None))
    pk = measured_peaks()
    byts = N * K + T * K * 3 + T * N * 2
    return {"op": "gemm_e4m3", "T": T, "N": N, "K": K, "fp8_ms": round(t8, 4), "bf16_ms": round(t16, 4),
            "fp8_TB/s": round(byts / t8 / 1e9, 2), "fp8_TFLOP/s": round(2.0 * T * N * K / t8 / 1e9, 1),
            "frac_bw": round(byts / t8 / 1e9 / (pk["hbm_gbs"] / 1e3), 3)}


def w4_case(T, N, K, group=128, once=False):
    """W4A16 int4 GEMM vs the library bf16 GEMM of the same shape (the
    int4 weight moves a quarter of the bytes; the roofline is the bytes of
    the int4 codes + scales + activations + output at the measured copy
    bandwidth)."""
    from ..ops import int4
    C = cuda_ext()
    x = torch.randn(T, K, device="cuda").bfloat16()
    w = (torch.randn(N, K, device="cuda") * 0.02).bfloat16()
    W = int4.quantize(w, group)
    y = torch.empty(T, N, device="cuda", dtype=torch.bfloat16)
    f4 = lambda: C.gemm_w4a16(y, x, W.qp, W.sz, N, group, None)  # noqa: E731
    if once:
        for _ in range(4):
            f4()
        torch.cuda.synchronize()
        return None
    t4 = _time(f4)
    t16 = _time(lambda: torch.matmul(x, w.t(), out=y))
    pk = measured_peaks()
    byts = W.qp.numel() + W.sz.numel() * 4 + T * K * 2 + T * N * 2
    return {"op": "gemm_w4a16", "T": T, "N": N, "K": K, "group": group, "w4_ms": round(t4, 4),
            "cublas_bf16_ms": round(t16, 4), "w4_TB/s": round(byts / t4 / 1e9, 2),
            "frac_bw": round(byts / t4 / 1e9 / (pk["hbm_gbs"] / 1e3), 3),
            "w4_TFLOP/s": round(2.0 * T * N * K / t4 / 1e9, 1)}


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
    ap.add_argument("op", choices=["gemm", "gemmchain", "decode", "prefill", "sweep", "step", "fp8",
                                       "w4"])
    ap.add_argument("--model", default="llama-2-7b")
    ap.add_argument("--eager", action="store_true")
    ap.add_argument("--shape", default=None)
    ap.add_argument("--splits", type=int, default=1)
    ap.add_argument("--once", action="store_true")
    ap.add_argument("--plan", default="-1,0,0", help="gemm2 plan,bn,splits (plan -1: automatic)")
    ap.add_argument("--kernel", default="gemm", choices=["gemm", "gemm2"],
                    help="gemm: the ops.linear dispatch; gemm2: the 2-SM kernel directly")
    ap.add_argument("--json", default=None)
    a = ap.parse_args(argv)
    if a.op == "sweep":
        res = sweep()
    elif a.op == "fp8":
        res = [fp8_case(*[int(v) for v in c.split("x")]) for c in
               (a.shape or "256x12288x4096,256x22016x4096,256x4096x11008,8192x12288x4096").split(",")]
        for r in res:
            print(json.dumps(r), flush=True)
        res = None
    elif a.op == "w4":
        res = []
        for c in (a.shape or "1x12288x4096,16x12288x4096,64x22016x4096,256x12288x4096,"
                             "256x4096x11008,1024x12288x4096,8192x12288x4096").split(","):
            r = w4_case(*[int(v) for v in c.split("x")], once=a.once)
            if r:
                print(json.dumps(r), flush=True)
                res.append(r)
    else:
        shp = [int(v) for v in a.shape.split(",")]
        if a.op == "gemm":
            res = gemm_case(*shp, once=a.once, kernel=a.kernel,
                            plan=tuple(int(v) for v in a.plan.split(",")))
        elif a.op == "gemmchain":
            res = gemm_chain_case(*shp)
        elif a.op == "step":
            res = step_case(*shp, model=a.model, eager=a.eager, once=a.once)
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
