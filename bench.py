"""Headline benchmark: output tokens/s of offline continuous batching on the
Llama-2-7B architecture (bf16, random init), tensor parallel over N GPUs.

Workload: 1000 requests of uniform-random token ids,
input lengths U[128, 1024], output lengths U[128, 512], seed 0, EOS ignored,
greedy decoding, KV block 16, gpu_memory_utilization 0.9.

One "step" is one engine iteration (schedule -> forward over the whole
continuous batch -> fused sampling -> scheduler update). The full workload
runs through the public API (``LLM.generate``): that is the end-to-end
number ("e2e"; every step copies its packed inputs host->device from pinned
memory and reads the sampled tokens back). Inside that run, once the batch
first fills to max_num_seqs and W more warm-up steps have run, K steps are
timed on the device (barrier + synchronize on both sides, CUDA events, max
over ranks): that is ``value``. Decode steps stream the 13.5 GB of weights
and the KV pool, far more than the 126 MB L2, so no L2 flush is needed.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
For N > 1 run under torchrun (one rank per GPU); rank 0 prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "output tok/s at Llama-2-7B/70B TP1-8 (max over ranks); p50 TTFT & TPOT"
MODEL = "llama-2-7b"


def workload(n_req: int, seed: int = 0, ins=(128, 1024), outs=(128, 512), vocab: int = 32000):
    """Uniform-random token ids; input / output lengths uniform in the closed
    ranges (a fixed length when lo == hi)."""
    rng = np.random.default_rng(seed)
    il = rng.integers(ins[0], ins[1] + 1, size=n_req)
    ol = rng.integers(outs[0], outs[1] + 1, size=n_req)
    prompts = [rng.integers(0, vocab, size=int(i)).tolist() for i in il]
    return prompts, [int(o) for o in ol]


# Named workloads (the model/config shapes of the benchmark plan). "llama2-7b"
# is the headline; the others exercise TP=8 on Llama-3-70B and MoE on Mixtral.
WORKLOADS = {
    "llama2-7b": dict(model="llama-2-7b", requests=1000, ins=(128, 1024), outs=(128, 512),
                      max_num_seqs=256, max_model_len=2048, vocab=32000,
                      desc="Llama-2-7B architecture (32L, H4096, 32 heads MHA, FFN 11008, V32000)"),
    "llama3-70b-decode": dict(model="llama-3-70b", requests=256, ins=(2048, 2048), outs=(256, 256),
                              max_num_seqs=256, max_model_len=2304, vocab=128256,
                              desc="Llama-3-70B architecture (80L, H8192, 64/8 heads, FFN 28672, "
                                   "V128256), decode-heavy: 256 x (2048 in, 256 out)"),
    "llama3-70b-prefill": dict(model="llama-3-70b", requests=64, ins=(4096, 4096), outs=(16, 16),
                               max_num_seqs=64, max_model_len=4112, vocab=128256,
                               desc="Llama-3-70B architecture, prefill-heavy: 64 x (4096 in, 16 out)"),
    "mixtral": dict(model="mixtral-8x7b", requests=512, ins=(256, 1024), outs=(256, 256),
                    max_num_seqs=256, max_model_len=1280, vocab=32000,
                    desc="Mixtral-8x7B architecture (32L, H4096, 32/8 heads, 8 experts top-2, "
                         "FFN 14336), experts split over the TP ranks"),
}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed window."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []
        self.th = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.th = threading.Thread(target=self._read, daemon=True)
        self.th.start()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.th:
            self.th.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [x.strip() for x in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        med = float(np.median(sm)) if sm else None
        return {"sm_mhz": med, "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


class HostProfile:
    """Diagnostic: wraps the engine's executor / sampler / scheduler calls
    with host timers, and records CUDA events at the start of each step's
    forward and after its sampling, so the GPU idle gap between steps (host
    work the GPU waits for) can be measured. Not used for the reported
    numbers."""

    def __init__(self, eng):
        import torch
        self.torch = torch
        self.t = {"schedule": 0.0, "execute_host": 0.0, "sample_host": 0.0, "update": 0.0,
                  "process": 0.0}
        self.n = 0
        self.ev = []  # (start_event, end_event) per step
        ex, sm, sch = eng.executor, eng.sampler, eng.scheduler
        orig_exec, orig_samp = ex.execute, sm.__call__
        orig_sched, orig_upd = sch.schedule, sch.update
        orig_proc = eng._process
        prof = self

        def execute(si):
            e0 = torch.cuda.Event(enable_timing=True)
            e0.record()
            t0 = time.perf_counter()
            out = orig_exec(si)
            prof.t["execute_host"] += time.perf_counter() - t0
            prof._start = e0
            return out

        class _S:
            def __call__(self_, *a, **k):
                t0 = time.perf_counter()
                out = orig_samp(*a, **k)
                prof.t["sample_host"] += time.perf_counter() - t0
                e1 = torch.cuda.Event(enable_timing=True)
                e1.record()
                prof.ev.append((prof._start, e1))
                prof.n += 1
                return out

            def __getattr__(self_, k):
                return getattr(sm, k)

        def timed(name, fn):
            def w(*a, **k):
                t0 = time.perf_counter()
                r = fn(*a, **k)
                prof.t[name] += time.perf_counter() - t0
                return r
            return w

        ex.execute = execute
        eng.sampler = _S()
        eng.scheduler = _Wrap(sch, schedule=timed("schedule", orig_sched),
                              update=timed("update", orig_upd))
        eng._process = timed("process", orig_proc)

    def report(self):
        self.torch.cuda.synchronize()
        gaps, busy = [], []
        for i, (s, e) in enumerate(self.ev):
            busy.append(s.elapsed_time(e))
            if i + 1 < len(self.ev):
                gaps.append(e.elapsed_time(self.ev[i + 1][0]))
        n = max(self.n, 1)
        return {"steps": self.n,
                "host_ms_per_step": {k: round(v / n * 1e3, 3) for k, v in self.t.items()},
                "gpu_step_ms_avg": round(sum(busy) / max(len(busy), 1), 3),
                "gpu_idle_gap_ms_avg": round(sum(gaps) / max(len(gaps), 1), 3)}


class _Wrap:
    def __init__(self, obj, **over):
        self._o = obj
        self.__dict__.update(over)

    def __getattr__(self, k):
        return getattr(self._o, k)


def reference_arm(args) -> None:
    msg = ("reference cannot be installed or run: its pyproject needs the maturin (Rust) build "
           "backend, absent offline, and its forward pass returns zeros / canned text "
           "(crates/swiftllm-models/src/layers/mod.rs:65-78, python/swiftllm/engine.py:351-384)")
    if int(os.environ.get("RANK", "0")) == 0:
        print(json.dumps({"impl": "reference", "unavailable": msg}))


def _model_bytes(mcfg) -> int:
    """bf16 bytes of the full (single-rank) model."""
    H, D, L = mcfg.hidden_size, mcfg.head_dim, mcfg.num_layers
    qkv = (mcfg.num_heads + 2 * mcfg.num_kv_heads) * D * H
    o = mcfg.num_heads * D * H
    mlp = 3 * mcfg.intermediate_size * H * max(1, mcfg.num_experts or 1)
    return 2 * (L * (qkv + o + mlp) + 2 * mcfg.vocab_size * H)


CHECK_LEN = 48   # prompt tokens of the TP logits check
CHECK_ROWS = 8   # last rows whose logits are compared


def tp_reference_logits(model: str, ekw: dict):
    """Rank 0, before the TP engine exists: the same dummy-initialised model
    on one GPU (no tensor parallelism, cuBLAS GEMMs) runs a CHECK_LEN-token
    prefill and returns the fp32 logits of its last CHECK_ROWS positions, or
    None when the model does not fit one GPU comfortably."""
    import torch
    from swiftllm_b200 import ops
    from swiftllm_b200.config import EngineConfig
    from swiftllm_b200.engine.llm_engine import prepare_config
    from swiftllm_b200.runtime.model_runner import ModelRunner, prefill_step_input
    cfg = EngineConfig(model=model, **dict(ekw, tensor_parallel_size=1))
    mcfg = prepare_config(cfg)
    if _model_bytes(mcfg) > 0.4 * torch.cuda.get_device_properties(0).total_memory:
        return None, None
    ops.set_gemm_backend("cublas")
    runner = ModelRunner(mcfg, cfg, torch.device("cuda", torch.cuda.current_device()), None,
                         cfg.max_model_len)
    runner.load_weights()
    ids = np.random.default_rng(1).integers(0, mcfg.vocab_size, size=CHECK_LEN).tolist()
    si = prefill_step_input(ids, cfg.block_size, CHECK_ROWS)
    runner.allocate_kv(si.max_blocks + 1, 0)
    logits = runner.execute(si).float().cpu()
    # the same single-GPU forward with our GEMMs: how far two correct bf16
    # forwards of these weights differ (the tolerance of the TP check)
    ops.set_gemm_backend("tcgen05")
    alt = runner.execute(si).float().cpu()
    runner.release()
    ops.set_gemm_backend(ops.DEFAULT_GEMM_BACKEND)
    return ids, (logits, alt)


def tp_logits_check(eng, ids, ref) -> dict:
    """One prefill step of the check prompt through the TP engine's executor
    (every rank runs it; blocks 0.. are free before any request) compared
    with the single-GPU logits."""
    import torch
    from swiftllm_b200.runtime.model_runner import prefill_step_input
    si = prefill_step_input(ids, eng.config.block_size, CHECK_ROWS)
    got = eng.executor.execute(si).float().cpu()
    ref, alt = ref
    err = (got - ref).abs().max().item()
    noise = (alt - ref).abs().max().item()
    scale = ref.abs().max().item()
    cos = torch.nn.functional.cosine_similarity(got, ref, dim=-1).min().item()
    cos_noise = torch.nn.functional.cosine_similarity(alt, ref, dim=-1).min().item()
    return {"vs": "tp1 single-GPU forward (cuBLAS GEMMs), same weights", "rows": CHECK_ROWS,
            "max_abs_err": round(err, 4), "ref_max_abs": round(scale, 4),
            "min_cosine": round(cos, 6),
            "tp1_tcgen05_vs_cublas": {"max_abs_err": round(noise, 4),
                                      "min_cosine": round(cos_noise, 6)},
            "ok": bool(err <= 2.0 * noise + 1e-3 * scale)}


def run_arm(args, wl, arm: str, rank: int, check=None):
    """One full run of the workload through LLM.generate with the given
    backend arm ("ours": tcgen05 GEMMs + fused NVLink reductions; "baseline":
    cuBLAS GEMMs + NCCL all-reduce, the same engine otherwise). Returns the
    result dict on rank 0, None on the other ranks. Leaves no device memory
    of the engine behind."""
    import gc
    import torch
    from swiftllm_b200 import LLM, SamplingParams, ops
    from swiftllm_b200.config import EngineConfig
    comm = args.comm if arm == "ours" else "nccl"
    ekw = dict(load_format="dummy", dtype="bfloat16", tensor_parallel_size=args.gpus,
               gpu_memory_utilization=0.9, block_size=16, max_num_seqs=args.max_num_seqs,
               enable_chunked_prefill=True, max_num_batched_tokens=8192,
               max_model_len=wl["max_model_len"], comm_backend=comm, seed=0,
               preemption_mode="recompute")
    os.environ["SWIFTLLM_CHANNEL"] = f"/swiftllm-bench-{os.environ.get('MASTER_PORT', '0')}-{arm}"
    if arm == "ours":
        ops.set_gemm_backend(args.gemm)
    if rank != 0:
        from swiftllm_b200.parallel.executor import run_worker_from_env
        run_worker_from_env(EngineConfig(model=args.model, **ekw))
        gc.collect()
        torch.cuda.empty_cache()
        return None

    prompts, out_lens = workload(args.requests, 0, wl["ins"], wl["outs"], wl["vocab"])
    sps = [SamplingParams(temperature=0.0, max_tokens=o, ignore_eos=True) for o in out_lens]
    t_init = time.time()
    llm = LLM(args.model, **ekw)
    eng = llm.llm_engine
    eng._ensure_initialized()
    init_s = time.time() - t_init
    check_res = tp_logits_check(eng, check[0], check[1]) if check is not None else None
    clocks = ClockSampler(int(os.environ.get("LOCAL_RANK", "0")))
    st = {"filled": None, "start": None, "stop": None, "tok": 0, "launch0": 0, "launches": 0}

    def hook(e):
        s = e.num_steps
        if st["filled"] is None and e.scheduler.num_running >= args.max_num_seqs:
            st["filled"] = s
        if st["filled"] is not None and st["start"] is None and s >= st["filled"] + args.warmup:
            clocks.start()
            e.executor.timer("start")
            st["start"] = s
            st["launch0"] = ops.LAUNCHES[0]
            return
        if st["start"] is not None and st["stop"] is None:
            st["tok"] += e.last_step_tokens
            if s >= st["start"] + args.steps:
                e.executor.timer("stop")
                st["stop"] = s
                st["launches"] = ops.LAUNCHES[0] - st["launch0"]

    eng.step_hook = hook
    prof = HostProfile(eng) if args.profile_host and arm == "ours" else None
    torch.cuda.synchronize()
    io_before = list(eng.io_bytes)
    steps_before = eng.num_steps
    t0 = time.perf_counter()
    outs = llm.generate(prompt_token_ids=prompts, sampling_params=sps, use_tqdm=False)
    torch.cuda.synchronize()
    e2e_s = time.perf_counter() - t0
    if st["start"] is not None and st["stop"] is None:  # workload ended inside the window
        eng.executor.timer("stop")
        st["stop"] = eng.num_steps
        st["launches"] = ops.LAUNCHES[0] - st["launch0"]
    clk = clocks.stop() if st["start"] is not None else {"sm_mhz": None, "reasons": ["no window"]}
    ms = eng.executor.timer("report") if st["start"] is not None else None
    n_out = sum(len(o.outputs[0].token_ids) for o in outs)
    steps_total = eng.num_steps - steps_before
    h2d = (eng.io_bytes[0] - io_before[0]) / max(steps_total, 1)
    d2h = (eng.io_bytes[1] - io_before[1]) / max(steps_total, 1)
    ttft = [o.metrics["ttft"] for o in outs if o.metrics and o.metrics["ttft"] is not None]
    tpot = [o.metrics["tpot"] for o in outs if o.metrics and o.metrics["tpot"] is not None]
    timed_steps = (st["stop"] - st["start"]) if st["start"] is not None else 0
    value = st["tok"] / (ms / 1e3) if ms else None
    res = {
        "value": round(value, 1) if value else None,
        "ms_per_step": round(ms / max(timed_steps, 1), 3) if ms else None,
        "steps": timed_steps,
        "e2e": {"value": round(n_out / e2e_s, 1),
                "unit": "output tokens/s (LLM.generate, whole workload)",
                "seconds": round(e2e_s, 2), "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h), "engine_steps": steps_total,
                "output_tokens": n_out},
        "p50_ttft_ms": round(float(np.median(ttft)) * 1e3, 1) if ttft else None,
        "p50_tpot_ms": round(float(np.median(tpot)) * 1e3, 2) if tpot else None,
        "gpu_launches": int(st["launches"]),
        "clocks": clk,
        "init_s": round(init_s, 1),
    }
    if check_res is not None:
        res["tp_check"] = check_res
    if prof is not None:
        res["host_profile"] = prof.report()
    llm.shutdown()
    del llm, eng, outs
    gc.collect()
    torch.cuda.empty_cache()
    return res


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--requests", type=int, default=None)
    ap.add_argument("--model", default=None)
    ap.add_argument("--workload", default="llama2-7b", choices=sorted(WORKLOADS))
    ap.add_argument("--max-num-seqs", type=int, default=None)
    ap.add_argument("--comm", default="fused", choices=["fused", "nccl"])
    ap.add_argument("--gemm", default="auto", choices=["auto", "tcgen05", "cublas"])
    ap.add_argument("--baseline", default="run", choices=["run", "skip"],
                    help="also run the cuBLAS + NCCL arm on the same workload (vs_baseline)")
    ap.add_argument("--profile-host", action="store_true",
                    help="report host phases and the GPU idle gap between steps (diagnostic)")
    args = ap.parse_args()
    wl = WORKLOADS[args.workload]
    args.model = args.model or wl["model"]
    args.requests = args.requests or wl["requests"]
    args.max_num_seqs = args.max_num_seqs or wl["max_num_seqs"]
    if args.impl == "reference":
        reference_arm(args)
        return
    args.warmup = max(args.warmup, 3)
    os.environ["SWIFTLLM_GEMM"] = args.gemm
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    if world > 1:
        from swiftllm_b200.parallel.comm import init_distributed
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        init_distributed(rank, world, "nccl")
    check = None
    if world > 1 and rank == 0:
        ids, ref = tp_reference_logits(args.model, dict(
            load_format="dummy", dtype="bfloat16", block_size=16, max_num_seqs=CHECK_ROWS,
            enable_chunked_prefill=True, max_num_batched_tokens=8192,
            max_model_len=wl["max_model_len"], seed=0, enforce_eager=True))
        check = (ids, ref) if ids is not None else None
    arms = ["baseline", "ours"] if args.baseline == "run" else ["ours"]
    results = {arm: run_arm(args, wl, arm, rank, check if arm == "ours" else None) for arm in arms}
    if rank == 0:
        r, b = results["ours"], results.get("baseline")
        vs = (round(r["value"] / b["value"], 3) if b and b.get("value") and r.get("value")
              else None)
        res = {
            "metric": METRIC,
            "value": r["value"],
            "unit": "output tokens/s",
            "n_gpus": args.gpus,
            "steps": r["steps"],
            "warmup": args.warmup,
            "ms_per_step": r["ms_per_step"],
            "higher_is_better": True,
            "scaling": "strong",
            "vs_baseline": vs,
            "dtype": "bf16",
            "data": "synthetic (uniform random token ids, random-init N(0,0.02) weights)",
            "config": {
                "model": wl["desc"],
                "workload": args.workload,
                "global_batch": args.max_num_seqs,
                "seq_len": f"in U[{wl['ins'][0]},{wl['ins'][1]}], out U[{wl['outs'][0]},{wl['outs'][1]}]",
                "requests": args.requests,
                "parallelism": f"tp{args.gpus}",
                "comm": args.comm if args.gpus > 1 else "none",
                "gemm": args.gemm,
                "l2": "no flush: each step streams weights + KV pool (>126 MB L2)",
                "window": f"{r['steps']} engine steps starting {args.warmup} steps after the batch "
                          f"first filled to {args.max_num_seqs} running sequences",
                "baseline_arm": "same engine and workload with cuBLAS GEMMs (torch.matmul) and "
                                "NCCL all-reduce / all-gather, run first in this process",
            },
            "e2e": r["e2e"],
            "p50_ttft_ms": r["p50_ttft_ms"],
            "p50_tpot_ms": r["p50_tpot_ms"],
            "gpu_launches": r["gpu_launches"],
            "clocks": r["clocks"],
            "init_s": r["init_s"],
        }
        if b is not None:
            res["baseline"] = {k: b[k] for k in ("value", "ms_per_step", "e2e", "p50_ttft_ms",
                                                 "p50_tpot_ms", "clocks")}
            res["e2e_vs_baseline"] = (round(r["e2e"]["value"] / b["e2e"]["value"], 3)
                                      if b["e2e"]["value"] else None)
        for k in ("tp_check", "host_profile"):
            if k in r:
                res[k] = r[k]
        print(json.dumps(res), flush=True)
    if world > 1:
        from swiftllm_b200.parallel.comm import teardown_distributed
        teardown_distributed()


if __name__ == "__main__":
    main()
