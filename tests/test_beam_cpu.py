"""Beam search on the CPU runner: width 1 equals greedy decoding, and a
width-3 search matches a plain-Python beam search that scores prefixes
through the same engine (top next-token log-probabilities of each prefix),
with the returned beams in score order and no KV blocks leaked."""

import numpy as np
import pytest
import torch

from swiftllm_b200 import LLM, SamplingParams

PROMPT = np.random.default_rng(7).integers(0, 32000, 23).tolist()


@pytest.fixture(scope="module")
def llm():
    return LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32", max_num_seqs=8,
               max_model_len=256)


def test_beam_width_one_is_greedy(llm):
    g = llm.generate(prompt_token_ids=[PROMPT], use_tqdm=False,
                     sampling_params=SamplingParams(temperature=0, max_tokens=6, ignore_eos=True))
    b = llm.generate(prompt_token_ids=[PROMPT], use_tqdm=False,
                     sampling_params=SamplingParams(temperature=0, max_tokens=6, ignore_eos=True,
                                                    use_beam_search=True))
    assert b[0].outputs[0].token_ids == g[0].outputs[0].token_ids


def _next_logprobs(model, prefix):
    """log-softmax of the next-token logits after ``prefix`` (fp32 CPU model
    with the engine's dummy weights)."""
    from swiftllm_b200.models.decoder import AttnMeta
    T = len(prefix)
    nb = (T + 15) // 16
    meta = AttnMeta(num_seqs=1, num_decode_seqs=0, num_tokens=T, max_q_len=T, max_seq_len=T,
                    positions=torch.arange(T, dtype=torch.int32),
                    slot_mapping=torch.arange(T, dtype=torch.int32),
                    q_start=torch.tensor([0, T], dtype=torch.int32),
                    seq_lens=torch.tensor([T], dtype=torch.int32),
                    block_tables=torch.arange(nb, dtype=torch.int32).view(1, nb),
                    logits_idx=torch.tensor([T - 1], dtype=torch.int32))
    cfg = model.cfg
    kv = torch.zeros(nb, cfg.num_layers, 2, model.local_kv_heads, 16, cfg.head_dim)
    with torch.no_grad():
        lg = model.compute_logits(model.forward(torch.tensor(prefix, dtype=torch.int32), meta, kv))
    return torch.log_softmax(lg[-1].double(), dim=-1)


def test_beam_width_three_matches_python_search(llm):
    W, steps = 3, 4
    sp = SamplingParams(temperature=0, max_tokens=steps, ignore_eos=True, use_beam_search=True,
                        n=W, best_of=W)
    out = llm.generate(prompt_token_ids=[PROMPT], sampling_params=sp, use_tqdm=False)[0]
    got = [(c.token_ids, c.cumulative_logprob) for c in out.outputs]
    assert len(got) == W
    scores = [cl / len(t) for t, cl in got]
    assert scores == sorted(scores, reverse=True)

    # reference: expand every live beam by its 2W best tokens, keep the W best
    from swiftllm_b200.models.config import load_config
    from swiftllm_b200.models.decoder import DecoderModel
    model = DecoderModel(load_config("tiny-llama"), torch.float32, "cpu")
    model.allocate()
    model.init_dummy(llm.llm_engine.config.seed)
    beams = [([], 0.0)]
    for _ in range(steps):
        cands = []
        for toks, cum in beams:
            v, i = _next_logprobs(model, PROMPT + toks).topk(2 * W)
            cands += [(toks + [int(t)], cum + float(x)) for x, t in zip(v, i)]
        cands.sort(key=lambda c: -c[1])
        beams = cands[:W]
    ref = sorted(beams, key=lambda c: -c[1] / len(c[0]))
    for (t, cl), (rt, rcl) in zip(got, ref):
        assert t == rt
        assert abs(cl - rcl) < 1e-3 * max(1.0, abs(rcl))
    # every beam's blocks went back to the pool
    bm = llm.llm_engine.block_manager
    assert bm.num_free_gpu_blocks == bm.num_gpu_blocks


def test_beam_finished_hypotheses_and_early_stop(llm):
    # make the greedy second token a stop token: hypotheses ending there
    # finish while the other beams go on
    g = llm.generate(prompt_token_ids=[PROMPT], use_tqdm=False,
                     sampling_params=SamplingParams(temperature=0, max_tokens=3, ignore_eos=True))
    stop_tok = g[0].outputs[0].token_ids[1]
    for early in (False, True):
        sp = SamplingParams(temperature=0, max_tokens=6, use_beam_search=True, n=2, best_of=3,
                            stop_token_ids=[stop_tok], early_stopping=early)
        out = llm.generate(prompt_token_ids=[PROMPT], sampling_params=sp, use_tqdm=False)[0]
        assert 1 <= len(out.outputs) <= 2
        assert any(c.token_ids[-1] == stop_tok and c.finish_reason.value == "stop"
                   for c in out.outputs) or all(len(c.token_ids) == 6 for c in out.outputs)
        bm = llm.llm_engine.block_manager
        assert bm.num_free_gpu_blocks == bm.num_gpu_blocks
