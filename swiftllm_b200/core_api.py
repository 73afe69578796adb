"""The low-level ``_core`` surface of SwiftLLM (RustEngine, RustBlockManager,
RustScheduler, RustSampler, cuda_* helpers) over this package's C++ core.

``import swiftllm._core`` resolves here, so code written against the
reference's type stubs (python/swiftllm/_core.pyi:8-136) keeps working.
Every class is a thin adapter: the work happens in the C++ extension
``swiftllm_b200._core`` (block manager, scheduler, Philox sampler) or in
LLMEngine (which runs the model, where the reference's step only schedules).

Dict-shaped arguments follow the stubs: ``config`` for RustEngine is
EngineConfig's fields by name; ``sampling_params`` is SamplingParams'
fields by name; ``step()`` returns one dict per finished or streamed
request: {"request_id", "token_ids", "text", "finished", "finish_reason"}.
"""

from __future__ import annotations

from typing import Any, Dict, List, Optional, Tuple

import numpy as np

from . import _core

__all__ = ["RustEngine", "RustBlockManager", "RustScheduler", "RustSampler", "cuda_available",
           "cuda_device_count", "cuda_get_device_properties", "cuda_synchronize"]


def _sampling_params(d: Optional[Dict[str, Any]]):
    from .config import SamplingParams
    return SamplingParams(**(d or {}))


class RustEngine:
    """Engine driven by dicts: add_request / abort_request / step."""

    def __init__(self, config: Dict[str, Any]) -> None:
        from .config import EngineConfig
        from .engine.llm_engine import LLMEngine
        cfg = dict(config)
        if "model" not in cfg:
            raise ValueError("config needs a 'model'")
        self._engine = LLMEngine(EngineConfig(**cfg))

    def add_request(self, request_id: str, prompt_token_ids: List[int],
                    sampling_params: Dict[str, Any]) -> None:
        self._engine.add_request(request_id, None, _sampling_params(sampling_params),
                                 prompt_token_ids=list(prompt_token_ids))

    def abort_request(self, request_id: str) -> None:
        self._engine.abort_request(request_id)

    def step(self) -> List[Dict[str, Any]]:
        out = []
        for o in self._engine.step():
            c = o.outputs[0] if o.outputs else None
            out.append({"request_id": o.request_id,
                        "token_ids": list(c.token_ids) if c else [],
                        "text": c.text if c else "",
                        "finished": o.finished,
                        "finish_reason": (getattr(c.finish_reason, "value", c.finish_reason)
                                          if c else None)})
        return out

    def get_num_unfinished_requests(self) -> int:
        return self._engine.get_num_unfinished_requests()

    def has_unfinished_requests(self) -> bool:
        return self._engine.has_unfinished_requests()

    def shutdown(self) -> None:
        self._engine.shutdown()


class RustBlockManager:
    """Paged-KV block allocator: blocks are counted per sequence."""

    def __init__(self, block_size: int, num_gpu_blocks: int, num_cpu_blocks: int) -> None:
        self._bm = _core.BlockManager(block_size, num_gpu_blocks, num_cpu_blocks, 0.0, False)
        self.block_size = block_size

    def allocate(self, seq_id: int, num_blocks: int) -> List[int]:
        """Grow ``seq_id``'s table to at least ``num_blocks`` blocks."""
        have = len(self._bm.get_block_table(seq_id)) if self._bm.has(seq_id) else 0
        if num_blocks > have and not self._bm.can_allocate(num_blocks - have):
            raise RuntimeError("out of KV blocks")
        ok, _ = self._bm.ensure_slots(seq_id, 0, num_blocks * self.block_size)
        if not ok:
            raise RuntimeError("out of KV blocks")
        return list(self._bm.get_block_table(seq_id))

    def free(self, seq_id: int) -> None:
        self._bm.free(seq_id)

    def can_allocate(self, num_blocks: int) -> bool:
        return self._bm.can_allocate(num_blocks)

    def get_block_table(self, seq_id: int) -> List[int]:
        return list(self._bm.get_block_table(seq_id)) if self._bm.has(seq_id) else []


class RustScheduler:
    """Continuous-batching scheduler over its own block manager.

    config keys: block_size (16), num_gpu_blocks (1024), num_cpu_blocks (0),
    max_num_seqs (256), max_num_batched_tokens (4096), max_model_len (4096),
    enable_chunked_prefill (True), policy ("fcfs" / "sjf" / "priority"),
    preemption ("recompute" / "swap").
    """

    def __init__(self, config: Dict[str, Any]) -> None:
        c = dict(config or {})
        self._bm = _core.BlockManager(int(c.get("block_size", 16)), int(c.get("num_gpu_blocks", 1024)),
                                      int(c.get("num_cpu_blocks", 0)), 0.01, False)
        sc = _core.SchedulerConfig()
        sc.max_num_seqs = int(c.get("max_num_seqs", 256))
        sc.max_num_batched_tokens = int(c.get("max_num_batched_tokens", 4096))
        sc.max_model_len = int(c.get("max_model_len", 4096))
        sc.enable_chunked_prefill = bool(c.get("enable_chunked_prefill", True))
        sc.policy = {"fcfs": _core.Policy.FCFS, "sjf": _core.Policy.SJF,
                     "priority": _core.Policy.PRIORITY}[str(c.get("policy", "fcfs"))]
        sc.preemption = {"recompute": _core.Preempt.RECOMPUTE,
                         "swap": _core.Preempt.SWAP}[str(c.get("preemption", "recompute"))]
        self._s = _core.Scheduler(sc, self._bm)
        self._batch = None
        self._swapped = set()

    def add_request(self, request_id: str, prompt_token_ids: List[int],
                    sampling_params: Dict[str, Any]) -> None:
        sp = _sampling_params(sampling_params)
        p = _core.GroupParams()
        p.n = sp.n
        p.max_tokens = sp.max_tokens
        p.min_tokens = sp.min_tokens
        p.ignore_eos = sp.ignore_eos
        p.stop_token_ids = list(sp.stop_token_ids or [])
        p.temperature = sp.temperature
        p.top_p = sp.top_p
        p.top_k = sp.top_k
        p.min_p = sp.min_p
        p.seed = -1 if sp.seed is None else int(sp.seed)
        self._s.add_request(request_id, np.asarray(prompt_token_ids, np.int32), p, 0.0)

    def _rid(self, seq: int) -> str:
        return self._s.group_info(self._s.seq_info(int(seq))["group"])["request_id"]

    def schedule(self) -> Tuple[List[str], List[str], List[str]]:
        """(scheduled request ids, preempted request ids, swapped-in ids)."""
        b = self._s.schedule(0.0)
        self._batch = b
        sched = list(dict.fromkeys(self._rid(s) for s in b.seq_ids))
        pre = [self._s.group_info(g)["request_id"] for g in b.preempted_groups
               if self._s.group_info(g) is not None]
        swapped_in = [r for r in sched if r in self._swapped]
        self._swapped.difference_update(swapped_in)
        if len(b.swap_out):
            self._swapped.update(pre)
        return sched, pre, swapped_in

    def update(self, outputs: List[Dict[str, Any]]) -> None:
        """outputs: {"request_id", "token_id"} per sampled row of the last
        schedule() (rows of requests not listed get token 0)."""
        b = self._batch
        if b is None:
            raise RuntimeError("update() before schedule()")
        by_rid = {o["request_id"]: int(o["token_id"]) for o in outputs}
        rows = [self._rid(b.seq_ids[r]) for r in b.sample_seq_row]
        toks = np.asarray([by_rid.get(r, 0) for r in rows], np.int32)
        self._s.update(b, toks, None, 0.0)
        self._batch = None

    def has_unfinished(self) -> bool:
        return self._s.has_unfinished()


class RustSampler:
    """One-row sampler (CPU, the same Philox stream and stage order as the
    GPU kernel). config: temperature, top_p, top_k, min_p, presence_penalty,
    frequency_penalty, repetition_penalty, seed."""

    def __init__(self, config: Dict[str, Any]) -> None:
        c = dict(config or {})
        self._p = _core.SampleParams(
            temperature=float(c.get("temperature", 1.0)), top_p=float(c.get("top_p", 1.0)),
            top_k=int(c.get("top_k", -1)), min_p=float(c.get("min_p", 0.0)),
            presence_penalty=float(c.get("presence_penalty", 0.0)),
            frequency_penalty=float(c.get("frequency_penalty", 0.0)),
            repetition_penalty=float(c.get("repetition_penalty", 1.0)))
        seed = c.get("seed")
        self._key = (0x5EED if seed is None else int(seed)) & 0xFFFFFFFFFFFFFFFF
        self._step = 0

    def sample(self, logits: List[float], token_ids: Optional[List[int]] = None) -> Tuple[int, float]:
        u = _core.philox_uniform(self._key, self._step & 0xFFFFFFFF, self._step >> 32)
        self._step += 1
        out = np.asarray(token_ids or [], np.int32)
        tok, lp = _core.sample_row(np.ascontiguousarray(np.asarray(logits, np.float32).reshape(-1)),
                                   self._p, u, np.zeros(0, np.int32), out)
        return int(tok), float(lp)


def cuda_available() -> bool:
    import torch
    return torch.cuda.is_available()


def cuda_device_count() -> int:
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def cuda_get_device_properties(device_id: int) -> Dict[str, Any]:
    import torch
    p = torch.cuda.get_device_properties(device_id)
    return {"name": p.name, "total_memory": p.total_memory,
            "multi_processor_count": p.multi_processor_count,
            "major": p.major, "minor": p.minor,
            "compute_capability": f"{p.major}.{p.minor}"}


def cuda_synchronize() -> None:
    import torch
    if torch.cuda.is_available():
        for d in range(torch.cuda.device_count()):
            torch.cuda.synchronize(d)
