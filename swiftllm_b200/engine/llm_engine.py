"""LLMEngine: the Python shell over the native core.

Each ``step()``: the C++ scheduler picks the batch (continuous batching,
chunked prefill, preemption) -> the executor runs the forward on every
tensor-parallel rank -> the fused GPU sampler draws tokens -> the C++ core
appends them and applies stop rules -> Python builds outputs only for
requests that stream, need stop strings or logprobs, or just finished.

Parity: python/swiftllm/engine.py:107-392 (LLMEngine add_request /
abort_request / step / has_unfinished_requests) and the Rust Engine
(crates/swiftllm-core/src/engine.rs: add_request :123-135, abort_request
:149-153, step :161-199, stats :259-267). The reference's step only
schedules and bumps a counter (engine.rs:188-198); this one runs the model.
"""

from __future__ import annotations

import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import numpy as np

from .. import _core
from ..config import EngineConfig, LoRARequest, PreemptionMode, SamplingParams, SchedulerPolicy
from ..outputs import CompletionOutput, FinishReason, RequestOutput, TokenLogprob
from ..utils.logging import get_logger
from ..utils import nvtx

log = get_logger(__name__)


@dataclass
class _Req:
    request_id: str
    prompt: Optional[str]
    prompt_ids: List[int]
    params: SamplingParams
    gid: int
    stream: bool = False
    texts: Dict[int, str] = field(default_factory=dict)       # seq -> text so far
    stop_reason: Dict[int, Any] = field(default_factory=dict)
    logprobs: Dict[int, List[TokenLogprob]] = field(default_factory=dict)
    finished_seqs: Dict[int, str] = field(default_factory=dict)
    done: bool = False
    arrival: float = 0.0
    beam_fin: List[Any] = field(default_factory=list)  # (penalised score, seq) of finished hypotheses


def prepare_config(c: EngineConfig):
    """Resolve the model and fill the derived engine settings (max_model_len,
    max_num_batched_tokens). Every tensor-parallel rank calls this on the same
    EngineConfig, so all ranks agree on shapes. Returns the ModelConfig."""
    from ..model_resolver import resolve_model
    from ..models.config import load_config
    if c.load_format != "dummy":
        c.model = resolve_model(c.model, download_dir=c.download_dir)
    mcfg = load_config(c.model)
    max_len = c.max_model_len or min(mcfg.max_position_embeddings, 4096)
    c.max_model_len = max_len
    if c.max_num_batched_tokens is None:
        c.max_num_batched_tokens = max(max_len, 8192) if not c.enable_chunked_prefill \
            else max(c.max_prefill_tokens, 2048)
    if not c.enable_chunked_prefill and c.max_num_batched_tokens < max_len:
        c.max_num_batched_tokens = max_len
    return mcfg


class LLMEngine:
    def __init__(self, config: EngineConfig):
        self.config = config
        self._initialized = False
        from ..utils.profiler import StepProfiler
        self._profiler = StepProfiler()
        self._reqs: Dict[str, _Req] = {}
        self._by_gid: Dict[int, _Req] = {}
        self._counter = 0
        self.tokenizer = None
        self.model_config = None
        self.executor = None
        self.scheduler = None
        self.block_manager = None
        self.sampler = None
        self.spec = None
        self._t_start = time.monotonic()
        self._gen_tokens = 0
        self._prompt_tokens = 0
        self._aborted: List[str] = []
        # instrumentation (bench): tokens of the last step, host<->device bytes
        # moved by steps (h2d, d2h), step count and an optional per-step hook
        self.last_step_tokens = 0
        self.io_bytes = [0, 0]
        self.num_steps = 0
        self.step_hook = None
        self._fatal: Optional[BaseException] = None  # a dead worker / peer: the engine is unusable

    # ------------------------------------------------------------ init
    def _ensure_initialized(self) -> None:
        if self._initialized:
            return
        from .tokenizer import load_tokenizer
        from ..parallel.executor import make_executor
        from ..sampling.batch import BatchSampler
        c = self.config
        self.model_config = prepare_config(c)
        mcfg = self.model_config
        path = c.model
        max_len = c.max_model_len
        tok_path = c.tokenizer if c.tokenizer and c.tokenizer != "" else path
        self.tokenizer = load_tokenizer(tok_path, mcfg.vocab_size, c.trust_remote_code)
        self.eos_token_id = getattr(self.tokenizer, "eos_token_id", None)
        if self.eos_token_id is None:
            self.eos_token_id = mcfg.eos_token_id
        if c.speculative_model:
            from .speculative import reserve_draft_memory
            reserve_draft_memory(c)
        self.executor = make_executor(mcfg, c)
        num_gpu, num_cpu = self.executor.num_gpu_blocks, self.executor.num_cpu_blocks
        self.block_manager = _core.BlockManager(c.block_size, num_gpu, num_cpu, c.watermark,
                                                c.enable_prefix_caching)
        sc = _core.SchedulerConfig()
        sc.max_num_seqs = c.max_num_seqs
        sc.max_num_batched_tokens = int(c.max_num_batched_tokens)
        sc.max_model_len = int(max_len)
        sc.enable_chunked_prefill = bool(c.enable_chunked_prefill)
        sc.policy = {SchedulerPolicy.FCFS: _core.Policy.FCFS, SchedulerPolicy.SJF: _core.Policy.SJF,
                     SchedulerPolicy.PRIORITY: _core.Policy.PRIORITY}[c.scheduler_policy]
        sc.preemption = (_core.Preempt.SWAP if c.preemption_mode == PreemptionMode.SWAP and num_cpu > 0
                         else _core.Preempt.RECOMPUTE)
        if c.speculative_model:
            sc.num_speculative_tokens = int(c.num_speculative_tokens)
        self.scheduler = _core.Scheduler(sc, self.block_manager)
        self.sampler = BatchSampler(mcfg.vocab_size, c.seed, self.executor.device)
        if c.speculative_model:
            from .speculative import SpeculativeDecoder
            self.spec = SpeculativeDecoder(self, c.speculative_model, c.num_speculative_tokens)
        self._initialized = True
        log.info("engine ready: %s, %d GPU blocks, %d CPU blocks, tp=%d", mcfg.name or path,
                 num_gpu, num_cpu, c.tensor_parallel_size)

    # ------------------------------------------------------------ requests
    def add_request(self, request_id: str, prompt: Optional[str] = None,
                    sampling_params: Optional[SamplingParams] = None,
                    prompt_token_ids: Optional[List[int]] = None,
                    lora_request: Optional[LoRARequest] = None,
                    arrival_time: Optional[float] = None, priority: int = 0,
                    stream: bool = False) -> None:
        self._ensure_initialized()
        if self._fatal is not None:
            raise self._fatal
        if request_id in self._reqs:
            raise ValueError(f"duplicate request id {request_id!r}")
        sp = sampling_params or SamplingParams()
        if prompt_token_ids is None:
            if prompt is None:
                raise ValueError("either prompt or prompt_token_ids is required")
            prompt_token_ids = list(self.tokenizer.encode(prompt))
        if sp.use_beam_search and sp.logprobs is not None:
            raise ValueError("beam search does not return per-token logprobs")
        gp = _core.GroupParams()
        # beam search: one sequence at admission; the beams are forked by
        # the engine's beam step (width max(n, best_of))
        gp.n = 1 if sp.use_beam_search else max(sp.n, sp.best_of)
        gp.max_tokens = sp.max_tokens
        gp.min_tokens = sp.min_tokens
        gp.ignore_eos = sp.ignore_eos
        gp.eos_token_id = int(self.eos_token_id) if self.eos_token_id is not None else -1
        gp.stop_token_ids = list(sp.stop_token_ids or [])
        gp.temperature = sp.temperature
        gp.top_p = sp.top_p
        gp.top_k = sp.top_k
        gp.min_p = sp.min_p
        gp.presence_penalty = sp.presence_penalty
        gp.frequency_penalty = sp.frequency_penalty
        gp.repetition_penalty = sp.repetition_penalty
        gp.seed = -1 if sp.seed is None else int(sp.seed)
        gp.priority = priority
        arrival = time.monotonic() if arrival_time is None else arrival_time
        ids = np.asarray(prompt_token_ids, dtype=np.int32)
        if ids.size and (ids.min() < 0 or ids.max() >= self.model_config.vocab_size):
            raise ValueError("prompt token id out of vocabulary range")
        gid = self.scheduler.add_request(request_id, ids, gp, arrival)
        r = _Req(request_id, prompt, list(map(int, prompt_token_ids)), sp, gid, stream=stream,
                 arrival=arrival)
        self._reqs[request_id] = r
        self._by_gid[gid] = r
        self._prompt_tokens += len(prompt_token_ids)

    def abort_request(self, request_id) -> None:
        ids = [request_id] if isinstance(request_id, str) else list(request_id)
        for rid in ids:
            r = self._reqs.get(rid)
            if r is None:
                continue
            self.scheduler.abort_request(rid)
            self._aborted.append(rid)

    def get_num_unfinished_requests(self) -> int:
        return len([r for r in self._reqs.values() if not r.done])

    def has_unfinished_requests(self) -> bool:
        return self.get_num_unfinished_requests() > 0

    # ------------------------------------------------------------ step
    def _history(self, sid: int):
        prompt = self.scheduler.seq_tokens(sid, False)
        info = self.scheduler.seq_info(sid)
        n = info["num_prompt"]
        return prompt[:n], prompt[n:]

    def step(self) -> List[RequestOutput]:
        """One engine iteration. If a tensor-parallel worker dies or a peer
        stops answering, every in-flight request is finished with
        finish_reason "abort" in this call's outputs and the engine raises
        that error on any later use."""
        self._ensure_initialized()
        if self._fatal is not None:
            raise self._fatal
        from ..parallel.failures import CommTimeoutError, WorkerDiedError
        try:
            outs = self._step()
            self._profiler.step()
            return outs
        except (WorkerDiedError, CommTimeoutError) as e:
            log.error("engine stopped: %s; aborting %d in-flight requests", e,
                      self.get_num_unfinished_requests())
            self._fatal = e
            outs = []
            for r in list(self._reqs.values()):
                if not r.done:
                    self.scheduler.abort_request(r.request_id)
                    outs.append(self._final_output(r, aborted=True))
            return outs

    def _expire(self) -> None:
        """Abort requests older than request_timeout_secs (0 disables)."""
        limit = float(getattr(self.config, "request_timeout_secs", 0) or 0)
        if limit <= 0:
            return
        now = time.monotonic()
        for r in self._reqs.values():
            if not r.done and r.request_id not in self._aborted and now - r.arrival > limit:
                log.warning("request %s timed out after %.0f s", r.request_id, now - r.arrival)
                self.abort_request(r.request_id)

    def _step(self) -> List[RequestOutput]:
        outs: List[RequestOutput] = []
        self._expire()
        for rid in self._aborted:
            r = self._reqs.get(rid)
            if r is not None and not r.done:
                outs.append(self._final_output(r, aborted=True))
        self._aborted = []
        if self.spec is not None:
            return outs + self.spec.step()
        with nvtx.range("schedule"):
            b = self.scheduler.schedule(time.monotonic())
        outs += self._rejected(b)
        if b.num_seqs == 0 and b.swap_in.size == 0 and b.swap_out.size == 0:
            return outs
        from ..runtime.model_runner import step_input_from_batch
        si = step_input_from_batch(b)
        want_lp_rows = self._wants_logprobs(b) if b.num_sample_rows else False
        beam_rows = self._beam_rows(b) if b.num_sample_rows else {}
        if self.config.tensor_parallel_size > 1 and b.num_sample_rows and not b.any_penalty \
                and not want_lp_rows and not beam_rows:
            temp = np.asarray(b.temperature)
            si.greedy = bool(np.all((temp <= 0.0) | (np.asarray(b.top_k) == 1)))
        logits = self.executor.execute(si)
        if b.num_sample_rows == 0:
            self.last_step_tokens = 0
            self.io_bytes[0] += si.ints.nbytes
            self.num_steps += 1
            if self.step_hook is not None:
                self.step_hook(self)
            return outs
        with nvtx.range("sample"):
            toks, lps = self.sampler(logits, b, self._history)
        want_lp = self._top_logprobs(logits, b, toks) if want_lp_rows else None
        if beam_rows:
            toks = np.array(toks, dtype=np.int32, copy=True)
            for rows in beam_rows.values():
                toks[rows] = -1  # handled by the beam step below
        res = self.scheduler.update(b, toks, lps, time.monotonic())
        ntok = len(res.token)
        outs += self._process(res, want_lp)
        if beam_rows:
            with nvtx.range("beam"):
                for gid, rows in beam_rows.items():
                    o, n = self._beam_step(gid, rows, logits, b)
                    outs += o
                    ntok += n
        self._gen_tokens += ntok
        self._account(si, b, ntok)
        return outs

    # ------------------------------------------------------------ beam search
    def _beam_rows(self, b) -> Dict[int, List[int]]:
        """Sample rows of beam-search groups in this batch, by group."""
        out: Dict[int, List[int]] = {}
        for i, g in enumerate(np.asarray(b.sample_group).tolist()):
            r = self._by_gid.get(int(g))
            if r is not None and r.params.use_beam_search:
                out.setdefault(int(g), []).append(i)
        return out

    @staticmethod
    def _beam_score(cum: float, n_out: int, length_penalty: float) -> float:
        return cum / (max(n_out, 1) ** length_penalty)

    def _beam_step(self, gid: int, rows: List[int], logits, b):
        """One beam-search step for group ``gid`` (its beams are ``rows`` of
        the batch): every beam proposes its 2W best next tokens, candidates
        are ranked by cumulative log-probability, the first W that do not end
        the sequence become the live beams, ending candidates ranked among
        the first W become finished hypotheses (scored cum / len^length_penalty).
        The group stops when no beam is live, or (early_stopping) once W
        hypotheses are finished, or when no live beam can still beat the
        worst of the W best finished ones. Returns (outputs, tokens appended)."""
        import torch
        r = self._by_gid[gid]
        sp = r.params
        W = max(sp.n, sp.best_of)
        lidx = torch.as_tensor([int(b.sample_logit_idx[i]) for i in rows], dtype=torch.long,
                               device=logits.device)
        lp = torch.log_softmax(logits.index_select(0, lidx).float(), dim=-1)
        kk = min(2 * W, lp.shape[-1])
        tv, ti = lp.topk(kk, dim=-1)
        tv, ti = tv.cpu().numpy(), ti.cpu().numpy()
        sids = [int(b.sample_target_seq[i]) for i in rows]
        info = {sid: self.scheduler.seq_info(sid) for sid in sids}
        eos = self.eos_token_id if not sp.ignore_eos else None
        stops = set(sp.stop_token_ids or [])
        cands = []
        for j, sid in enumerate(sids):
            cum = float(info[sid]["cum_logprob"])
            for q in range(kk):
                cands.append((cum + float(tv[j, q]), sid, int(ti[j, q]), float(tv[j, q])))
        cands.sort(key=lambda c: -c[0])
        live, fin = [], []
        for rank, (score, sid, tok, v) in enumerate(cands):
            n_out = int(info[sid]["num_output"]) + 1
            ends = n_out > sp.min_tokens and ((eos is not None and tok == eos) or tok in stops)
            if ends:
                if rank < W:
                    fin.append((sid, tok, v, n_out, score))
            elif len(live) < W:
                live.append((sid, tok, v))
            if len(live) == W:
                break
        res = self.scheduler.beam_update(gid, [c[0] for c in live], [c[1] for c in live],
                                         [c[2] for c in live], [c[0] for c in fin],
                                         [c[1] for c in fin], [c[2] for c in fin], time.monotonic())
        new_seqs = np.asarray(res.seq).tolist()
        for k, c in enumerate(fin):
            r.beam_fin.append((self._beam_score(c[4], c[3], sp.length_penalty), new_seqs[k]))
        r.beam_fin.sort(key=lambda x: -x[0])
        del r.beam_fin[W:]
        # stopping rules
        info_g = self.scheduler.group_info(gid)
        live_now = [s for s in (info_g["seqs"] if info_g else [])
                    if self.scheduler.seq_info(s)["status"] == "running"]
        stop = False
        if live_now and len(r.beam_fin) >= W:
            if sp.early_stopping:
                stop = True
            else:
                best_live = max(float(self.scheduler.seq_info(s)["cum_logprob"]) for s in live_now)
                n_out = max(int(self.scheduler.seq_info(s)["num_output"]) for s in live_now)
                stop = self._beam_score(best_live, n_out, sp.length_penalty) <= r.beam_fin[-1][0]
        if stop:
            for s in live_now:
                self.scheduler.finish_seq(s, "abort")
        info_g = self.scheduler.group_info(gid)
        done = info_g is None or all(self.scheduler.seq_info(s)["status"] not in
                                     ("running", "waiting", "swapped") for s in info_g["seqs"])
        outs = []
        if done and not r.done:
            outs.append(self._final_output(r))
        elif r.stream:
            outs.append(self._make_output(r, final=False))
        return outs, len(res.token)

    def _rejected(self, b) -> List[RequestOutput]:
        outs = []
        for g in b.preempted_groups:
            if g < 0:  # rejected: prompt can never fit the KV pool
                r = self._by_gid.get(-g)
                if r is not None:
                    log.warning("request %s rejected: prompt exceeds KV cache capacity", r.request_id)
                    outs.append(self._final_output(r))
        return outs

    def _wants_logprobs(self, b) -> bool:
        return any(self._by_gid[g].params.logprobs for g in set(np.asarray(b.sample_group).tolist())
                   if g in self._by_gid)

    def _account(self, si, b, ntok: int) -> None:
        self.last_step_tokens = ntok
        self.io_bytes[0] += si.ints.nbytes + si.logits_idx.nbytes + 28 * int(b.num_sample_rows)
        self.io_bytes[1] += 8 * int(b.num_sample_rows)
        self.num_steps += 1
        if self.step_hook is not None:
            self.step_hook(self)

    def _top_logprobs(self, logits, b, toks):
        import torch
        lidx = torch.from_numpy(np.asarray(b.sample_logit_idx, dtype=np.int64)).to(logits.device)
        groups = np.asarray(b.sample_group)
        n = max((self._by_gid[g].params.logprobs or 0) for g in groups if g in self._by_gid)
        lp = torch.log_softmax(logits.index_select(0, lidx).float(), dim=-1)
        top_v, top_i = lp.topk(max(n, 1), dim=-1)
        chosen = lp.gather(1, torch.from_numpy(toks.astype(np.int64)).to(lp.device).view(-1, 1))
        return top_v.cpu().numpy(), top_i.cpu().numpy(), chosen.view(-1).cpu().numpy()

    def _decode(self, ids) -> str:
        return self.tokenizer.decode(list(map(int, ids)), skip_special_tokens=True)

    def _process(self, res, want_lp) -> List[RequestOutput]:
        outs: List[RequestOutput] = []
        groups = res.group
        seqs = res.seq
        toks = res.token
        rows = res.row
        touched = set()
        for j in range(len(groups)):
            r = self._by_gid.get(int(groups[j]))
            if r is None:
                continue
            sp = r.params
            if not (sp.stop or r.stream or sp.logprobs is not None):
                continue
            sid = int(seqs[j])
            if sp.logprobs is not None and want_lp is not None:
                tv, ti, ch = want_lp
                row = int(rows[j])
                lst = r.logprobs.setdefault(sid, [])
                lst.append(TokenLogprob(int(toks[j]), self._decode([toks[j]]), float(ch[row]),
                                        bytes=None))
                top = r.__dict__.setdefault("top_logprobs", {}).setdefault(sid, [])
                top.append({int(ti[row, q]): float(tv[row, q]) for q in range(sp.logprobs)})
            if sp.stop:
                text = self._decode(self.scheduler.seq_tokens(sid, True))
                for s in sp.stop:
                    k = text.find(s)
                    if k >= 0:
                        r.texts[sid] = text[:k + len(s)] if sp.include_stop_str_in_output else text[:k]
                        r.stop_reason[sid] = s
                        self.scheduler.finish_seq(sid, "stop")
                        break
            touched.add(r.request_id)
        finished = set(int(g) for g in res.finished_groups)
        # groups finished by stop strings (finish_seq) are not in finished_groups
        for rid in list(touched):
            r = self._reqs[rid]
            if r.gid in finished:
                continue
            info = self.scheduler.group_info(r.gid)
            if info is not None and all(self.scheduler.seq_info(s)["status"] not in
                                        ("running", "waiting", "swapped") for s in info["seqs"]):
                finished.add(r.gid)
        for gid in finished:
            r = self._by_gid.get(gid)
            if r is not None and not r.done:
                outs.append(self._final_output(r))
                touched.discard(r.request_id)
        for rid in touched:
            r = self._reqs.get(rid)
            if r is not None and r.stream and not r.done:
                outs.append(self._make_output(r, final=False))
        return outs

    def _make_output(self, r: _Req, final: bool, aborted: bool = False) -> RequestOutput:
        info = self.scheduler.group_info(r.gid)
        comps: List[CompletionOutput] = []
        seq_ids = info["seqs"] if info else []
        for idx, sid in enumerate(seq_ids):
            si = self.scheduler.seq_info(sid)
            ids = self.scheduler.seq_tokens(sid, True).tolist()
            text = r.texts.get(sid)
            if text is None:
                text = self._decode(ids)
            status = si["status"]
            fr = None
            if aborted or status == "abort":
                fr = FinishReason.ABORT
            elif status == "stop":
                fr = FinishReason.STOP
            elif status == "length":
                fr = FinishReason.LENGTH
            stop_reason = r.stop_reason.get(sid)
            if fr == FinishReason.STOP and stop_reason is None and ids:
                stop_reason = ids[-1] if ids[-1] != self.eos_token_id else None
            comps.append(CompletionOutput(
                index=idx, text=text, token_ids=ids,
                cumulative_logprob=float(si["cum_logprob"]),
                logprobs=r.logprobs.get(sid), finish_reason=fr if final or fr else None,
                stop_reason=stop_reason))
        if r.params.use_beam_search:
            # beams: the best finished hypotheses (and beams cut by the
            # length limit) by length-penalised score; beams stopped early
            # or dropped are not results
            lp = r.params.length_penalty
            comps = [c for c in comps if c.finish_reason != FinishReason.ABORT or aborted]
            comps.sort(key=lambda c: -self._beam_score(c.cumulative_logprob or 0.0,
                                                        len(c.token_ids), lp))
            comps = comps[: r.params.n]
            for i, c in enumerate(comps):
                c.index = i
        elif final and r.params.best_of > r.params.n and len(comps) > r.params.n:
            comps.sort(key=lambda c: -(c.cumulative_logprob or 0.0))
            comps = comps[: r.params.n]
            for i, c in enumerate(comps):
                c.index = i
        metrics = None
        if info:
            arr, ft, fin = info["arrival"], info["first_token"], info["finished"]
            if fin < 0 and final:
                fin = time.monotonic()
            n_out = max((len(c.token_ids) for c in comps), default=0)
            metrics = {
                "arrival_time": arr, "first_scheduled_time": info["first_scheduled"],
                "first_token_time": ft, "finished_time": fin if final else -1.0,
                "ttft": (ft - arr) if ft >= 0 else None,
                "tpot": ((fin - ft) / (n_out - 1)) if final and ft >= 0 and n_out > 1 else None,
                "prompt_tokens": len(r.prompt_ids), "completion_tokens": sum(len(c.token_ids) for c in comps),
                "num_preemptions": info["num_preemptions"],
            }
        return RequestOutput(request_id=r.request_id, prompt=r.prompt, prompt_token_ids=r.prompt_ids,
                             outputs=comps, finished=final, metrics=metrics)

    def _final_output(self, r: _Req, aborted: bool = False) -> RequestOutput:
        out = self._make_output(r, final=True, aborted=aborted)
        r.done = True
        self.scheduler.release_group(r.gid)
        self._reqs.pop(r.request_id, None)
        self._by_gid.pop(r.gid, None)
        return out

    # ------------------------------------------------------------ stats
    def stats(self) -> Dict[str, Any]:
        self._ensure_initialized()
        st = self.scheduler.stats()
        bm = self.block_manager
        el = max(time.monotonic() - self._t_start, 1e-9)
        return {
            "num_running": self.scheduler.num_running,
            "num_waiting": self.scheduler.num_waiting,
            "num_swapped": self.scheduler.num_swapped,
            "completed_requests": st.finished,
            "aborted_requests": st.aborted,
            "throughput_tps": self._gen_tokens / el,
            "gpu_block_utilization": 1.0 - bm.num_free_gpu_blocks / max(bm.num_gpu_blocks, 1),
            "cpu_block_utilization": (1.0 - bm.num_free_cpu_blocks / bm.num_cpu_blocks)
            if bm.num_cpu_blocks else 0.0,
            "free_gpu_blocks": bm.num_free_gpu_blocks,
            "free_cpu_blocks": bm.num_free_cpu_blocks,
            "prefill_tokens": st.prefill_tokens,
            "decode_tokens": st.decode_tokens,
            "forward_passes": st.steps,
            "num_preemptions": st.num_preemptions,
            "prefix_cache_hit_rate": (st.prefix_cache_hit_tokens / st.prefix_cache_query_tokens)
            if st.prefix_cache_query_tokens else 0.0,
        }

    def shutdown(self) -> None:
        self._profiler.close()
        if self.executor is not None:
            self.executor.shutdown()
            self.executor = None

    def __del__(self):
        try:
            self.shutdown()
        except Exception:
            pass
