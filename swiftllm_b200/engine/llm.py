"""User-facing offline (``LLM``) and online (``AsyncLLM``) APIs.

Parity: python/swiftllm/engine.py:395-696 (LLM.__init__ / generate / encode
/ get_tokenizer, AsyncLLM.generate / abort, create_engine, generate). Extra
keyword arguments accepted: ``prompt_token_ids=`` on ``generate`` and any
EngineConfig field (``load_format="dummy"``, ``max_num_seqs``, ...).

``AsyncLLM`` drives one engine thread: requests enter through the native
RequestQueue (csrc/core/request_queue.h), the thread steps the engine while
work exists and hands each request's outputs to its asyncio queue. (The
reference polls ``step()`` from every request coroutine, engine.py:626-654,
which serialises concurrent requests.)
"""

from __future__ import annotations

import asyncio
import itertools
import threading
import time
import uuid
from typing import Any, AsyncIterator, Dict, List, Optional, Union

from .. import _core
from ..config import DataType, EngineConfig, LoRARequest, QuantizationMethod, SamplingParams
from ..outputs import RequestOutput
from .llm_engine import LLMEngine


def _engine_config(model: str, kwargs: Dict[str, Any]) -> EngineConfig:
    fields = EngineConfig.__dataclass_fields__
    unknown = [k for k in kwargs if k not in fields]
    if unknown:
        raise TypeError(f"unknown engine options: {unknown}")
    return EngineConfig(model=model, **kwargs)


class LLM:
    def __init__(self, model: str, tokenizer: Optional[str] = None, dtype: str = "auto",
                 quantization: Optional[str] = None, download_dir: Optional[str] = None,
                 max_model_len: Optional[int] = None, tensor_parallel_size: int = 1,
                 gpu_memory_utilization: float = 0.90, swap_space: float = 4.0,
                 trust_remote_code: bool = False, seed: int = 0, **kwargs):
        self.config = _engine_config(model, dict(
            tokenizer=tokenizer, dtype=DataType(dtype),
            quantization=QuantizationMethod(quantization) if quantization else QuantizationMethod.NONE,
            download_dir=download_dir, max_model_len=max_model_len,
            tensor_parallel_size=tensor_parallel_size,
            gpu_memory_utilization=gpu_memory_utilization, swap_space=swap_space,
            trust_remote_code=trust_remote_code, seed=seed, **kwargs))
        self._engine = LLMEngine(self.config)
        self._counter = itertools.count(1)

    @property
    def llm_engine(self) -> LLMEngine:
        return self._engine

    def _rid(self) -> str:
        return f"req-{next(self._counter)}-{uuid.uuid4().hex[:8]}"

    def generate(self, prompts: Union[str, List[str], None] = None,
                 sampling_params: Optional[Union[SamplingParams, List[SamplingParams]]] = None,
                 use_tqdm: bool = True, lora_request: Optional[LoRARequest] = None,
                 prompt_token_ids: Optional[List[List[int]]] = None) -> List[RequestOutput]:
        if prompts is None and prompt_token_ids is None:
            raise ValueError("prompts or prompt_token_ids is required")
        if isinstance(prompts, str):
            prompts = [prompts]
        n = len(prompts) if prompts is not None else len(prompt_token_ids)
        if prompt_token_ids is not None and prompts is not None and len(prompt_token_ids) != n:
            raise ValueError("prompts and prompt_token_ids differ in length")
        if sampling_params is None:
            sampling_params = [SamplingParams() for _ in range(n)]
        elif isinstance(sampling_params, SamplingParams):
            sampling_params = [sampling_params] * n
        if len(sampling_params) != n:
            raise ValueError(f"Number of sampling params ({len(sampling_params)}) must match "
                             f"number of prompts ({n})")
        rids = []
        for i in range(n):
            rid = self._rid()
            rids.append(rid)
            self._engine.add_request(
                rid, prompt=prompts[i] if prompts is not None else None,
                sampling_params=sampling_params[i],
                prompt_token_ids=prompt_token_ids[i] if prompt_token_ids is not None else None,
                lora_request=lora_request)
        pbar = None
        if use_tqdm:
            try:
                from tqdm import tqdm
                pbar = tqdm(total=n, desc="Generating")
            except ImportError:
                pbar = None
        outs: Dict[str, RequestOutput] = {}
        while self._engine.has_unfinished_requests():
            for o in self._engine.step():
                if o.finished:
                    outs[o.request_id] = o
                    if pbar is not None:
                        pbar.update(1)
        if pbar is not None:
            pbar.close()
        return [outs[r] for r in rids]

    def encode(self, prompts: Union[str, List[str]]) -> List[List[int]]:
        self._engine._ensure_initialized()
        if isinstance(prompts, str):
            prompts = [prompts]
        return [list(self._engine.tokenizer.encode(p)) for p in prompts]

    def get_tokenizer(self):
        self._engine._ensure_initialized()
        return self._engine.tokenizer

    def shutdown(self) -> None:
        self._engine.shutdown()


class AsyncLLM:
    def __init__(self, model: str, tokenizer: Optional[str] = None, **kwargs):
        self.config = _engine_config(model, dict(tokenizer=tokenizer, **kwargs))
        self._engine = LLMEngine(self.config)
        self._counter = itertools.count(1)
        self._queue = _core.RequestQueue(0, True, 0.0)
        self._pending: Dict[int, tuple] = {}
        self._handles = itertools.count(1)
        self._streams: Dict[str, tuple] = {}
        self._aborts: List[str] = []
        self._lock = threading.Lock()
        self._wake = threading.Event()
        self._stop = False
        self._thread: Optional[threading.Thread] = None
        self._error: Optional[BaseException] = None
        self._stats: Dict[str, Any] = {}
        self._stats_t = 0.0

    @property
    def engine(self) -> LLMEngine:
        return self._engine

    def _rid(self) -> str:
        return f"async-req-{next(self._counter)}-{uuid.uuid4().hex[:8]}"

    def start(self) -> None:
        if self._thread is None:
            self._engine._ensure_initialized()
            self._thread = threading.Thread(target=self._loop, name="swiftllm-engine", daemon=True)
            self._thread.start()

    def _loop(self) -> None:
        eng = self._engine
        try:
            while not self._stop:
                for e in self._queue.dequeue_batch(1 << 30):
                    with self._lock:
                        args = self._pending.pop(e.handle, None)
                    if args is None:
                        continue
                    rid, prompt, sp, ids, prio = args
                    try:
                        eng.add_request(rid, prompt=prompt, sampling_params=sp,
                                        prompt_token_ids=ids, priority=prio, stream=True)
                    except Exception as ex:  # deliver the error to the caller
                        self._deliver(rid, ex)
                with self._lock:
                    aborts, self._aborts = self._aborts, []
                if aborts:
                    eng.abort_request(aborts)
                if not eng.has_unfinished_requests():
                    self._wake.wait(0.05)
                    self._wake.clear()
                    continue
                for out in eng.step():
                    self._deliver(out.request_id, out)
                now = time.monotonic()
                if now - self._stats_t > 0.25:
                    snap = eng.stats()
                    with self._lock:
                        self._stats = snap
                    self._stats_t = now
        except BaseException as ex:  # engine failure ends every stream
            self._error = ex
            with self._lock:
                rids = list(self._streams)
            for rid in rids:
                self._deliver(rid, ex)

    def _deliver(self, rid: str, item) -> None:
        with self._lock:
            s = self._streams.get(rid)
        if s is None:
            return
        loop, q = s
        loop.call_soon_threadsafe(q.put_nowait, item)

    async def generate(self, prompt: Optional[str] = None,
                       sampling_params: Optional[SamplingParams] = None,
                       request_id: Optional[str] = None,
                       lora_request: Optional[LoRARequest] = None,
                       prompt_token_ids: Optional[List[int]] = None,
                       priority: int = 0) -> AsyncIterator[RequestOutput]:
        if self._error is not None:
            raise RuntimeError("engine stopped") from self._error
        self.start()
        sp = sampling_params or SamplingParams()
        rid = request_id or self._rid()
        q: asyncio.Queue = asyncio.Queue()
        with self._lock:
            self._streams[rid] = (asyncio.get_running_loop(), q)
            h = next(self._handles)
            self._pending[h] = (rid, prompt, sp, prompt_token_ids, priority)
        self._queue.enqueue(rid, h, priority)
        self._wake.set()
        try:
            while True:
                item = await q.get()
                if isinstance(item, BaseException):
                    raise item
                yield item
                if item.finished:
                    return
        finally:
            with self._lock:
                self._streams.pop(rid, None)
                if rid not in self._aborts:
                    self._aborts.append(rid)  # no-op if it already finished
            self._wake.set()

    def stats(self) -> Dict[str, Any]:
        """Engine counters (a snapshot the engine thread refreshes every
        250 ms; read directly when the thread is not running)."""
        if self._thread is None:
            self._engine._ensure_initialized()
            return self._engine.stats()
        with self._lock:
            return dict(self._stats)

    async def abort(self, request_id: str) -> None:
        with self._lock:
            self._aborts.append(request_id)
        self._wake.set()

    def shutdown(self) -> None:
        self._stop = True
        self._wake.set()
        if self._thread is not None:
            self._thread.join(timeout=10)
        self._engine.shutdown()


def create_engine(config: Union[EngineConfig, Dict[str, Any]]) -> LLMEngine:
    if isinstance(config, dict):
        config = EngineConfig.from_dict(config)
    return LLMEngine(config)


def generate(model: str, prompts: Union[str, List[str]],
             sampling_params: Optional[SamplingParams] = None, **kwargs) -> List[RequestOutput]:
    llm = LLM(model=model, **kwargs)
    return llm.generate(prompts, sampling_params)
