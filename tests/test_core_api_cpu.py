"""The ``swiftllm._core`` surface (RustEngine / RustBlockManager /
RustScheduler / RustSampler / cuda_*) on CPU."""

import numpy as np

from swiftllm import _core as C


def test_rust_engine_generates():
    eng = C.RustEngine({"model": "tiny-llama", "load_format": "dummy", "device": "cpu",
                        "dtype": "float32", "max_model_len": 128})
    eng.add_request("a", [1, 2, 3, 4], {"temperature": 0.0, "max_tokens": 5, "ignore_eos": True})
    eng.add_request("b", [9, 8, 7], {"temperature": 0.0, "max_tokens": 3, "ignore_eos": True})
    eng.abort_request("b")
    done = {}
    for _ in range(50):
        for o in eng.step():
            if o["finished"]:
                done[o["request_id"]] = o
        if not eng.has_unfinished_requests():
            break
    assert eng.get_num_unfinished_requests() == 0
    assert len(done["a"]["token_ids"]) == 5 and done["a"]["finish_reason"] == "length"
    eng.shutdown()


def test_rust_block_manager():
    bm = C.RustBlockManager(16, 8, 0)
    t = bm.allocate(1, 3)
    assert len(t) == 3 and bm.get_block_table(1) == t
    assert bm.can_allocate(5) and not bm.can_allocate(6)
    bm.free(1)
    assert bm.get_block_table(1) == [] and bm.can_allocate(8)


def test_rust_scheduler_runs_requests_to_completion():
    s = C.RustScheduler({"block_size": 16, "num_gpu_blocks": 64, "max_num_seqs": 4,
                         "max_num_batched_tokens": 64})
    s.add_request("x", list(range(40)), {"max_tokens": 3, "ignore_eos": True})
    s.add_request("y", list(range(10)), {"max_tokens": 2, "ignore_eos": True})
    seen = set()
    for _ in range(20):
        sched, pre, swapped = s.schedule()
        seen.update(sched)
        s.update([{"request_id": r, "token_id": 5} for r in sched])
        if not s.has_unfinished():
            break
    assert seen == {"x", "y"} and not s.has_unfinished()


def test_rust_sampler_and_cuda_helpers():
    logits = np.zeros(10, np.float32)
    logits[7] = 5.0
    tok, lp = C.RustSampler({"temperature": 0.0}).sample(logits.tolist())
    assert tok == 7 and lp < 0
    a = C.RustSampler({"temperature": 1.0, "top_k": 3, "seed": 11})
    b = C.RustSampler({"temperature": 1.0, "top_k": 3, "seed": 11})
    r = np.random.default_rng(0).normal(size=50).astype(np.float32).tolist()
    assert [a.sample(r)[0] for _ in range(5)] == [b.sample(r)[0] for _ in range(5)]
    assert isinstance(C.cuda_available(), bool) and C.cuda_device_count() >= 0
    C.cuda_synchronize()
