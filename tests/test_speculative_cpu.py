"""Speculative decoding through the engine (CPU, fp32 tiny models).

Greedy requests must produce exactly the tokens of plain decoding, with
n-gram drafts and with a draft model; sampled requests finish with the
requested lengths. The core's draft bookkeeping (append / rollback /
update_multi) is checked directly."""

import numpy as np
import pytest

from swiftllm_b200 import LLM, SamplingParams, _core


def _gen(spec=None, k=4, prompts=None, sp=None, **kw):
    llm = LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32",
              max_model_len=256, speculative_model=spec, num_speculative_tokens=k, **kw)
    outs = llm.generate(prompt_token_ids=prompts, sampling_params=sp, use_tqdm=False)
    return llm, [o.outputs[0].token_ids for o in outs]


REP = [[11, 12, 13, 14, 15, 16] * 6, [7, 8, 9] * 10, list(range(100, 130)), [42] * 20]


def test_ngram_greedy_equals_plain():
    sp = SamplingParams(temperature=0, max_tokens=40, ignore_eos=True)
    _, plain = _gen(None, prompts=REP, sp=sp)
    llm, spec = _gen("ngram", prompts=REP, sp=sp)
    assert spec == plain
    st = llm.llm_engine.spec.stats
    assert st["proposed"] > 0
    # a repetitive context keeps repeating under random weights often enough
    assert st["emitted"] > st["steps"]


def test_draft_model_greedy_equals_plain():
    sp = SamplingParams(temperature=0, max_tokens=24, ignore_eos=True)
    prompts = REP[:2] + [list(range(5, 40))]
    _, plain = _gen(None, prompts=prompts, sp=sp)
    llm, spec = _gen("tiny-llama", prompts=prompts, sp=sp)
    assert spec == plain
    st = llm.llm_engine.spec.stats
    # the draft is the target itself: (almost) every draft is accepted
    assert st["accepted"] >= 0.9 * st["proposed"] > 0


@pytest.mark.parametrize("spec", ["ngram", "tiny-llama"])
def test_sampled_spec_lengths(spec):
    sps = [SamplingParams(temperature=0.9, top_p=0.95, top_k=50, max_tokens=20, ignore_eos=True,
                          seed=1),
           SamplingParams(temperature=0, max_tokens=15, ignore_eos=True),
           SamplingParams(temperature=1.0, max_tokens=9, ignore_eos=True, stop=["zz"])]
    _, outs = _gen(spec, prompts=REP[:3], sp=sps)
    assert [len(o) for o in outs] == [20, 15, 9]


def test_spec_respects_max_tokens_and_eos():
    sp = SamplingParams(temperature=0, max_tokens=7, ignore_eos=True)
    _, outs = _gen("ngram", k=6, prompts=REP, sp=sp)
    assert all(len(o) == 7 for o in outs)
    _, plain = _gen(None, prompts=[REP[0]], sp=SamplingParams(temperature=0, max_tokens=12,
                                                             ignore_eos=True))
    stop_tok = plain[0][5]
    sp2 = SamplingParams(temperature=0, max_tokens=12, stop_token_ids=[stop_tok])
    _, outs = _gen("ngram", prompts=[REP[0]], sp=sp2)
    assert outs[0] == plain[0][:plain[0].index(stop_tok) + 1]


def test_core_draft_bookkeeping():
    bm = _core.BlockManager(4, 32, 0, 0.0, False)
    sc = _core.SchedulerConfig()
    sc.num_speculative_tokens = 3
    s = _core.Scheduler(sc, bm)
    gp = _core.GroupParams()
    gp.max_tokens = 10
    gp.ignore_eos = True
    s.add_request("a", np.arange(6, dtype=np.int32), gp, 0.0)
    b = s.schedule(0.0)
    s.update(b, np.array([50], np.int32))
    sid = int(s.decode_ready_seqs()[0])
    s.append_tokens(sid, [60, 61, 62])
    b = s.schedule(0.0)
    assert list(b.q_len) == [4] and b.num_sample_rows == 1
    # positions 6..9 computed; table must cover the reserved extra slots too
    assert len(bm.get_block_table(sid)) * 4 >= 10 + 3
    s.rollback(sid, 3)
    assert s.seq_info(sid)["num_computed"] == 6 and s.seq_info(sid)["num_draft"] == 0
    res = s.update_multi(b, np.array([60, 61, 70], np.int32), np.array([3], np.int32))
    assert list(res.token) == [60, 61, 70]
    info = s.seq_info(sid)
    assert info["num_tokens"] == 10 and info["num_computed"] == 9
    assert list(s.decode_ready_seqs()) == [sid]
    b = s.schedule(0.0)
    assert list(b.q_len) == [1] and list(b.positions) == [9]
    # max_tokens cuts a multi-token append short
    res = s.update_multi(b, np.array([1, 2, 3, 4, 5, 6, 7], np.int32), np.array([7], np.int32))
    assert len(res.token) == 6 and list(res.finished_groups)  # 4 + 6 = max_tokens
