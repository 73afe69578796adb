"""Engine behaviour on the CPU runner: config validation, text prompts,
stop strings / tokens, n and best_of, abort, AsyncLLM streaming, and
scheduler features (chunked prefill, prefix caching, preemption) that must
not change greedy outputs."""

import asyncio

import numpy as np
import pytest

from swiftllm_b200 import AsyncLLM, EngineConfig, LLM, SamplingParams
from swiftllm_b200.config import PreemptionMode


def _llm(**kw):
    base = dict(load_format="dummy", device="cpu", dtype="float32", max_num_seqs=8,
                max_model_len=256)
    base.update(kw)
    return LLM("tiny-llama", **base)


PROMPTS = [np.random.default_rng(1).integers(0, 32000, n).tolist() for n in (20, 37, 50, 9)]
GREEDY = SamplingParams(temperature=0, max_tokens=12, ignore_eos=True)


@pytest.fixture(scope="module")
def ref_tokens():
    llm = _llm()
    return [o.outputs[0].token_ids for o in
            llm.generate(prompt_token_ids=PROMPTS, sampling_params=GREEDY, use_tqdm=False)]


def test_sampling_params_validation():
    with pytest.raises(ValueError):
        SamplingParams(temperature=-1)
    with pytest.raises(ValueError):
        SamplingParams(top_p=1.5)
    with pytest.raises(ValueError):
        SamplingParams(top_k=0)
    with pytest.raises(ValueError):
        SamplingParams(max_tokens=0)
    with pytest.raises(ValueError):
        SamplingParams(n=3, best_of=2)
    assert SamplingParams(n=3).best_of == 3
    assert SamplingParams(stop="x").stop == ["x"]
    d = SamplingParams(temperature=0.5).to_dict()
    assert SamplingParams.from_dict(d).temperature == 0.5


def test_engine_config(monkeypatch):
    with pytest.raises(ValueError):
        EngineConfig(model="m", block_size=12)
    with pytest.raises(ValueError):
        EngineConfig(model="m", gpu_memory_utilization=0)
    c = EngineConfig.from_dict({"model": "m", "preemption_mode": "recompute", "junk": 1})
    assert c.preemption_mode == PreemptionMode.RECOMPUTE and c.tokenizer == "m"
    monkeypatch.setenv("SWIFTLLM_MAX_NUM_SEQS", "7")
    assert EngineConfig(model="m").max_num_seqs == 7
    assert EngineConfig(model="m").to_dict()["scheduler_policy"] == "fcfs"


def test_chunked_prefill_same_tokens(ref_tokens):
    llm = _llm(enable_chunked_prefill=True, max_num_batched_tokens=16)
    got = [o.outputs[0].token_ids for o in
           llm.generate(prompt_token_ids=PROMPTS, sampling_params=GREEDY, use_tqdm=False)]
    assert got == ref_tokens


def test_prefix_caching_same_tokens(ref_tokens):
    llm = _llm(enable_prefix_caching=True)
    a = [o.outputs[0].token_ids for o in
         llm.generate(prompt_token_ids=PROMPTS, sampling_params=GREEDY, use_tqdm=False)]
    b = [o.outputs[0].token_ids for o in
         llm.generate(prompt_token_ids=PROMPTS, sampling_params=GREEDY, use_tqdm=False)]
    assert a == ref_tokens and b == ref_tokens
    assert llm.llm_engine.stats()["prefix_cache_hit_rate"] > 0


@pytest.mark.parametrize("mode", ["recompute", "swap"])
def test_preemption_same_tokens(mode):
    # 7 blocks of 16 tokens cannot hold the growing sequences: preemption must
    # kick in and outputs must be unchanged
    sp = SamplingParams(temperature=0, max_tokens=40, ignore_eos=True)
    ref = [o.outputs[0].token_ids for o in
           _llm().generate(prompt_token_ids=PROMPTS, sampling_params=sp, use_tqdm=False)]
    llm = _llm(num_gpu_blocks_override=7, preemption_mode=mode, watermark=0.0)
    outs = llm.generate(prompt_token_ids=PROMPTS, sampling_params=sp, use_tqdm=False)
    assert [o.outputs[0].token_ids for o in outs] == ref
    assert llm.llm_engine.stats()["num_preemptions"] > 0


def test_text_prompt_stop_strings_and_tokens():
    llm = _llm()
    out = llm.generate(["Hello world"], SamplingParams(temperature=0, max_tokens=8,
                                                       ignore_eos=True), use_tqdm=False)[0]
    text = out.outputs[0].text
    assert out.prompt == "Hello world" and len(out.outputs[0].token_ids) == 8
    first = out.outputs[0].token_ids[2]
    o2 = llm.generate(["Hello world"], SamplingParams(temperature=0, max_tokens=8,
                                                      stop_token_ids=[first]), use_tqdm=False)[0]
    assert o2.outputs[0].token_ids[-1] == first and o2.outputs[0].finish_reason.value == "stop"
    if len(text) > 3:
        stop = text[2:4]
        o3 = llm.generate(["Hello world"], SamplingParams(temperature=0, max_tokens=8, stop=[stop],
                                                          ignore_eos=True), use_tqdm=False)[0]
        assert stop not in o3.outputs[0].text and o3.outputs[0].finish_reason.value == "stop"


def test_n_best_of_and_logprobs():
    llm = _llm()
    sp = SamplingParams(temperature=1.0, max_tokens=5, n=2, best_of=4, seed=7, logprobs=2,
                        ignore_eos=True)
    out = llm.generate(prompt_token_ids=[PROMPTS[0]], sampling_params=sp, use_tqdm=False)[0]
    assert len(out.outputs) == 2
    cl = [c.cumulative_logprob for c in out.outputs]
    assert cl[0] >= cl[1]
    assert len(out.outputs[0].logprobs) == 5
    assert out.metrics["completion_tokens"] == 10  # the n returned sequences


def test_abort_and_metrics():
    llm = _llm()
    eng = llm.llm_engine
    eng.add_request("a", prompt_token_ids=PROMPTS[0], sampling_params=GREEDY)
    eng.add_request("b", prompt_token_ids=PROMPTS[1], sampling_params=GREEDY)
    eng.step()
    eng.abort_request("a")
    outs = {}
    while eng.has_unfinished_requests():
        for o in eng.step():
            outs[o.request_id] = o
    assert outs["a"].outputs[0].finish_reason.value == "abort"
    assert outs["b"].outputs[0].finish_reason.value == "length"
    m = outs["b"].metrics
    assert m["ttft"] >= 0 and m["tpot"] >= 0 and m["prompt_tokens"] == len(PROMPTS[1])


def test_async_streaming():
    llm = AsyncLLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32",
                   max_num_seqs=8, max_model_len=256)

    async def run():
        async def one(i):
            seen = []
            async for o in llm.generate(prompt_token_ids=PROMPTS[i],
                                        sampling_params=SamplingParams(temperature=0, max_tokens=6,
                                                                       ignore_eos=True)):
                seen.append(len(o.outputs[0].token_ids))
            return seen
        return await asyncio.gather(*(one(i) for i in range(3)))

    res = asyncio.run(run())
    llm.shutdown()
    for seen in res:
        assert seen[-1] == 6 and seen == sorted(seen)


def test_rejects_bad_prompts():
    llm = _llm()
    with pytest.raises(ValueError):
        llm.generate(prompt_token_ids=[[40000]], sampling_params=GREEDY, use_tqdm=False)
    with pytest.raises(ValueError):
        llm.generate(prompt_token_ids=[list(range(300))], sampling_params=GREEDY, use_tqdm=False)


def test_alibi_model_generates_cpu():
    """A model with ALiBi position bias (no RoPE) runs through the engine, and
    the head slopes follow the ALiBi formula (2^-1 .. 2^-8 for 8 heads)."""
    import torch
    from swiftllm_b200.ops import reference as ref
    a = LLM("tiny-llama-alibi", load_format="dummy", device="cpu", dtype="float32", max_num_seqs=4,
            max_model_len=256)
    out = a.generate(prompt_token_ids=PROMPTS[:2], sampling_params=GREEDY, use_tqdm=False)
    assert all(len(o.outputs[0].token_ids) == 12 for o in out)
    s = ref.alibi_slopes(8)
    assert torch.allclose(s, torch.tensor([2.0 ** (-i) for i in range(1, 9)]))


def test_step_profiler_writes_trace(tmp_path, monkeypatch):
    # SWIFTLLM_PROFILE records a window of engine steps with torch.profiler
    monkeypatch.setenv("SWIFTLLM_PROFILE", str(tmp_path))
    monkeypatch.setenv("SWIFTLLM_PROFILE_SKIP", "2")
    monkeypatch.setenv("SWIFTLLM_PROFILE_STEPS", "3")
    from swiftllm_b200 import LLM, SamplingParams
    llm = LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32", max_model_len=128)
    llm.generate(prompt_token_ids=[[1, 2, 3, 4]], use_tqdm=False,
                 sampling_params=SamplingParams(temperature=0, max_tokens=8, ignore_eos=True))
    assert (tmp_path / "trace.json").stat().st_size > 0
    assert "Name" in (tmp_path / "summary.txt").read_text()
