"""Native core (C++) on CPU: block manager, scheduler, request queue,
sampler oracle, speculative helpers.

Re-expresses the reference's Rust unit tests as specifications:
block_manager.rs:562-621, scheduler/mod.rs:530-575,
continuous_batching.rs:560-576, request_queue.rs:411-506,
sampling/mod.rs:399-484, strategies.rs:445-518, speculative.rs:386-431,
kv_cache.rs:305-320."""

import threading
import time

import numpy as np
import pytest

from swiftllm_b200 import _core


# ------------------------------------------------------------ block manager
def test_block_math_and_refcounts():
    bm = _core.BlockManager(16, 100, 10, 0.0, False)
    assert bm.blocks_needed(100) == 7 and bm.blocks_needed(16) == 1 and bm.blocks_needed(17) == 2
    t = bm.allocate(1, 100)
    assert len(t) == 7 and bm.num_free_gpu_blocks == 93
    bm.fork(1, 2)
    assert all(bm.refcount(b) == 2 for b in t)
    bm.free(1)
    assert bm.num_free_gpu_blocks == 93 and all(bm.refcount(b) == 1 for b in t)
    bm.free(2)
    assert bm.num_free_gpu_blocks == 100


def test_copy_on_write_on_shared_partial_block():
    bm = _core.BlockManager(16, 10, 0, 0.0, False)
    bm.allocate(1, 20)
    bm.fork(1, 2)
    ok, cow = bm.ensure_slots(2, 20, 21)
    assert ok and cow.shape == (1, 2)
    src, dst = cow[0]
    assert src == bm.get_block_table(1)[1] and dst == bm.get_block_table(2)[1]
    assert bm.get_block_table(1)[0] == bm.get_block_table(2)[0]


def test_out_of_blocks_and_watermark():
    bm = _core.BlockManager(16, 10, 0, 0.2, False)
    assert bm.watermark_blocks == 2
    assert bm.can_allocate(8, True) and not bm.can_allocate(9, True) and bm.can_allocate(10, False)
    bm.allocate(1, 16 * 10)
    ok, _ = bm.ensure_slots(1, 160, 161)
    assert not ok


def test_swap_roundtrip():
    bm = _core.BlockManager(16, 8, 8, 0.0, False)
    t = bm.allocate(1, 40)
    m = bm.swap_out(1)
    assert m.shape == (3, 2) and list(m[:, 0]) == t and bm.num_free_gpu_blocks == 8
    assert bm.is_swapped(1) and bm.can_swap_in(1)
    m2 = bm.swap_in(1)
    assert m2.shape == (3, 2) and bm.num_free_cpu_blocks == 8
    assert list(m2[:, 0]) == list(m[:, 1])


def test_prefix_cache_hits():
    bm = _core.BlockManager(4, 8, 0, 0.0, True)
    toks = np.arange(13, dtype=np.int32)
    bm.allocate(1, 13)
    bm.register_full_blocks(1, toks, 13)
    assert bm.num_cached_blocks() == 3
    bm.free(1)
    assert bm.count_cached_blocks(toks) == 3
    assert bm.allocate_cached_prefix(2, toks, 3) == 12
    other = toks.copy()
    other[9] = 99
    assert bm.count_cached_blocks(other) == 2


# ------------------------------------------------------------ scheduler
def _sched(num_blocks=64, max_seqs=8, budget=64, chunked=True, policy=None, preempt=None,
           cpu_blocks=0, max_len=256, caching=False):
    bm = _core.BlockManager(4, num_blocks, cpu_blocks, 0.0, caching)
    sc = _core.SchedulerConfig()
    sc.max_num_seqs = max_seqs
    sc.max_num_batched_tokens = budget
    sc.max_model_len = max_len
    sc.enable_chunked_prefill = chunked
    if policy is not None:
        sc.policy = policy
    if preempt is not None:
        sc.preemption = preempt
    return _core.Scheduler(sc, bm), bm


def _gp(max_tokens=4, **kw):
    p = _core.GroupParams()
    p.max_tokens = max_tokens
    p.ignore_eos = True
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def _run_step(s, now=0.0, token=7):
    b = s.schedule(now)
    toks = np.full(b.num_sample_rows, token, dtype=np.int32)
    return b, s.update(b, toks, None, now)


def test_admission_finish_and_abort():
    s, bm = _sched()
    s.add_request("a", np.arange(10, dtype=np.int32), _gp(3), 0.0)
    s.add_request("b", np.arange(6, dtype=np.int32), _gp(2), 0.0)
    assert s.num_waiting == 2
    b, r = _run_step(s)
    assert b.num_seqs == 2 and b.num_tokens == 16 and s.num_running == 2
    assert list(b.q_len) == [10, 6] and b.num_decode_seqs == 0
    b, r = _run_step(s)
    assert b.num_decode_seqs == 2 and b.num_tokens == 2
    assert len(r.finished_groups) == 1
    assert s.abort_request("a")
    assert not s.has_unfinished() and bm.num_free_gpu_blocks == 64


def test_slot_mapping_and_positions():
    s, bm = _sched()
    s.add_request("a", np.arange(6, dtype=np.int32), _gp(3), 0.0)
    b = s.schedule(0.0)
    tab = bm.get_block_table(int(b.seq_ids[0]))
    assert list(b.positions) == list(range(6))
    assert list(b.slot_mapping) == [tab[p // 4] * 4 + p % 4 for p in range(6)]
    assert list(b.input_ids) == list(range(6))
    assert b.block_tables.shape == (1, 2)


def test_chunked_prefill_and_decode_first():
    s, _ = _sched(budget=16)
    s.add_request("long", np.arange(40, dtype=np.int32), _gp(2), 0.0)
    b, r = _run_step(s)
    assert b.num_tokens == 16 and b.num_sample_rows == 0
    b, r = _run_step(s)
    assert b.num_tokens == 16 and b.num_sample_rows == 0
    s.add_request("short", np.arange(5, dtype=np.int32), _gp(2), 0.0)
    b, r = _run_step(s)
    # the last 8 prompt tokens of "long" plus all 5 of "short": both sample
    assert b.num_tokens == 13 and b.num_sample_rows == 2
    b, r = _run_step(s)
    assert b.num_decode_seqs >= 1


def test_no_chunking_requires_whole_prompt():
    s, _ = _sched(budget=256, chunked=False)
    s.add_request("a", np.arange(200, dtype=np.int32), _gp(1), 0.0)
    s.add_request("b", np.arange(100, dtype=np.int32), _gp(1), 0.0)
    b, _ = _run_step(s)
    assert b.num_seqs == 1 and b.num_tokens == 200


def test_policies():
    for pol, expect in ((_core.Policy.FCFS, "x"), (_core.Policy.SJF, "y"),
                        (_core.Policy.PRIORITY, "y")):
        s, _ = _sched(max_seqs=1, policy=pol)
        s.add_request("x", np.arange(4, dtype=np.int32), _gp(10, priority=0), 0.0)
        s.add_request("y", np.arange(4, dtype=np.int32), _gp(2, priority=5), 0.0)
        b = s.schedule(0.0)
        info = s.group_info(int(b.sample_group[0]))
        assert info["request_id"] == expect, pol


def test_preemption_recompute_and_swap():
    for mode, cpu in ((_core.Preempt.RECOMPUTE, 0), (_core.Preempt.SWAP, 64)):
        s, bm = _sched(num_blocks=10, max_seqs=4, budget=64, preempt=mode, cpu_blocks=cpu)
        s.add_request("a", np.arange(8, dtype=np.int32), _gp(20), 0.0)
        s.add_request("b", np.arange(8, dtype=np.int32), _gp(20), 1.0)
        _run_step(s)
        done = False
        swapped = 0
        for _ in range(200):
            b, r = _run_step(s)
            swapped += b.swap_out.shape[0]
            if not s.has_unfinished():
                done = True
                break
        assert done
        assert s.stats().num_preemptions > 0
        if mode == _core.Preempt.SWAP:
            assert swapped > 0
        assert bm.num_free_gpu_blocks == 10


def test_n_greater_than_one_forks_with_shared_prompt():
    s, bm = _sched()
    s.add_request("a", np.arange(6, dtype=np.int32), _gp(3, n=3), 0.0)
    b = s.schedule(0.0)
    assert b.num_sample_rows == 3 and list(b.sample_target_seq).count(-1) == 2
    s.update(b, np.array([1, 2, 3], dtype=np.int32), None, 0.0)
    info = s.group_info(int(b.sample_group[0]))
    assert len(info["seqs"]) == 3
    outs = sorted(int(s.seq_tokens(q)[0]) for q in info["seqs"])
    assert outs == [1, 2, 3]
    b2 = s.schedule(0.0)
    assert b2.num_decode_seqs == 3 and b2.copies.shape[0] >= 2  # copy-on-write of the last block


def test_stop_tokens_eos_min_tokens():
    s, _ = _sched()
    p = _gp(10, eos_token_id=2, ignore_eos=False, min_tokens=2, stop_token_ids=[9])
    s.add_request("a", np.arange(4, dtype=np.int32), p, 0.0)
    _, r = _run_step(s, token=2)  # eos before min_tokens: ignored
    assert not r.finished_groups
    _, r = _run_step(s, token=2)
    assert r.finished_groups
    s.add_request("b", np.arange(4, dtype=np.int32), p, 0.0)
    _run_step(s, token=5)
    _, r = _run_step(s, token=9)
    gid = r.finished_groups[0]
    assert s.seq_info(s.group_info(gid)["seqs"][0])["status"] == "stop"


def test_ttft_is_first_token_time():
    s, _ = _sched(budget=8)
    s.add_request("a", np.arange(20, dtype=np.int32), _gp(2), 0.0)
    _run_step(s, now=1.0)
    _run_step(s, now=2.0)
    b, r = _run_step(s, now=3.0)
    info = s.group_info(int(b.sample_group[0]))
    assert info["first_scheduled"] == 1.0 and info["first_token"] == 3.0


def test_prefix_caching_through_scheduler():
    s, bm = _sched(caching=True)
    prompt = np.arange(20, dtype=np.int32)
    s.add_request("a", prompt, _gp(1), 0.0)
    _run_step(s)
    s.add_request("b", prompt, _gp(1), 0.0)
    b, _ = _run_step(s)
    assert b.num_tokens == 4  # 16 of 20 tokens reused
    assert s.stats().prefix_cache_hit_tokens == 16


def test_rejects_bad_requests():
    s, _ = _sched(max_len=16)
    with pytest.raises(ValueError):
        s.add_request("a", np.arange(16, dtype=np.int32), _gp(1), 0.0)
    s.add_request("b", np.arange(4, dtype=np.int32), _gp(1), 0.0)
    with pytest.raises(ValueError):
        s.add_request("b", np.arange(4, dtype=np.int32), _gp(1), 0.0)


# ------------------------------------------------------------ request queue
def test_request_queue_priority_full_close_timeouts():
    q = _core.RequestQueue(3, True, 0.05)
    assert q.enqueue("a", 1, 0) == _core.EnqueueStatus.OK
    assert q.enqueue("b", 2, 5) == _core.EnqueueStatus.OK
    assert q.enqueue("c", 3, 0) == _core.EnqueueStatus.OK
    assert q.enqueue("d", 4, 0) == _core.EnqueueStatus.FULL
    assert q.dequeue(0.0).id == "b"
    assert q.remove("c") and not q.remove("zz")
    q.stop_accepting()
    assert q.enqueue("e", 5, 0) == _core.EnqueueStatus.CLOSED
    q.start_accepting()
    time.sleep(0.08)
    timed = q.drain_timeouts()
    assert [e.id for e in timed] == ["a"] and len(q) == 0
    st = q.stats()
    assert st.rejected == 2 and st.timed_out == 1


def test_request_queue_blocking_dequeue():
    q = _core.RequestQueue()
    got = []
    th = threading.Thread(target=lambda: got.append(q.dequeue(2.0)))
    th.start()
    time.sleep(0.05)
    q.enqueue("x", 7, 0)
    th.join()
    assert got[0].id == "x" and got[0].handle == 7
    assert q.dequeue(0.01) is None


# ------------------------------------------------------------ sampler oracle
def test_greedy_and_logprob():
    lg = np.array([0.1, 3.0, 1.0, -2.0], dtype=np.float32)
    t, lp = _core.sample_row(lg, _core.SampleParams(temperature=0.0), 0.5)
    assert t == 1
    ref = lg[1] - lg.max() - np.log(np.exp(lg - lg.max()).sum())
    assert abs(lp - ref) < 1e-5


def test_top_k_support_and_temperature_statistics():
    rng = np.random.default_rng(42)
    lg = rng.normal(size=100).astype(np.float32)
    top5 = set(np.argsort(-lg)[:5].tolist())
    p = _core.SampleParams(temperature=1.0, top_k=5)
    seen = {_core.sample_row(lg, p, _core.philox_uniform(42, i))[0] for i in range(500)}
    assert seen <= top5 and len(seen) >= 3
    cold = _core.SampleParams(temperature=0.05)
    hits = sum(_core.sample_row(lg, cold, _core.philox_uniform(7, i))[0] == int(np.argmax(lg))
               for i in range(200))
    assert hits > 190


def test_top_p_keeps_crossing_token_and_min_p():
    lg = np.log(np.array([0.5, 0.3, 0.15, 0.05], dtype=np.float32))
    p = _core.SampleParams(temperature=1.0, top_p=0.6)
    seen = {_core.sample_row(lg, p, _core.philox_uniform(1, i))[0] for i in range(300)}
    assert seen == {0, 1}
    pm = _core.SampleParams(temperature=1.0, min_p=0.5)
    seen = {_core.sample_row(lg, pm, _core.philox_uniform(2, i))[0] for i in range(300)}
    assert seen == {0, 1}


def test_penalties():
    lg = np.array([2.0, -1.0, 1.0], dtype=np.float32)
    p = _core.SampleParams(temperature=0.0, repetition_penalty=4.0)
    t, _ = _core.sample_row(lg, p, 0.0, np.array([0], np.int32), np.zeros(0, np.int32))
    assert t == 2
    p2 = _core.SampleParams(temperature=0.0, frequency_penalty=1.0, presence_penalty=0.5)
    t, _ = _core.sample_row(lg, p2, 0.0, np.zeros(0, np.int32), np.array([0, 0], np.int32))
    assert t == 2


def test_philox_known_answer():
    # Random123 known-answer vector for philox4x32-10, zero key and counter
    assert _core.philox_block(0, 0, 0, 0, 0) == (0x6627E8D5, 0xE169C58D, 0xBC57AC4C, 0x9B00DBD8)


# ------------------------------------------------------------ speculative helpers
def test_spec_verify_accepts_identical_and_rejects_impossible():
    V = 5
    dp = np.full((2, V), 0.2, dtype=np.float32)
    tp = np.full((3, V), 0.2, dtype=np.float32)
    n, toks = _core.spec_verify(dp, tp, np.array([1, 3], np.int32), np.full(5, 0.5, np.float32))
    assert n == 2 and toks[:2] == [1, 3] and len(toks) == 3
    tp2 = tp.copy()
    tp2[0] = [0.0, 0.0, 1.0, 0.0, 0.0]
    n, toks = _core.spec_verify(dp, tp2, np.array([1, 3], np.int32), np.full(5, 0.5, np.float32))
    assert n == 0 and toks == [2]


def test_ngram_and_adaptive_k():
    ng = _core.NgramSpeculator(3, 8)
    ctx = np.array([1, 2, 3, 4, 5, 9, 9, 1, 2, 3], np.int32)
    assert ng.propose(ctx, 3) == [4, 5, 9]
    ak = _core.AdaptiveK(5, 1, 10, 0.7)
    for _ in range(30):
        ak.update(5, 5)
    assert ak.k == 10 and ak.acceptance_rate == 1.0
    for _ in range(200):
        ak.update(5, 0)
    assert ak.k < 10


def test_kv_bytes():
    from swiftllm_b200.models.config import ModelConfig
    c = ModelConfig(num_layers=1, num_kv_heads=8, head_dim=128)
    assert c.kv_cache_bytes_per_token(2) == 4096  # K + V: 2 x 8 x 128 x 2 B
    assert 16 * c.kv_cache_bytes_per_token(2) == 65536


def test_row_keys_vectorised_matches_mix_key():
    # per-row Philox keys / counters: seeded rows use (seed, step index),
    # the others the engine key with (step, row)
    import numpy as np
    from swiftllm_b200.parallel.dummy_init import mix_key
    from swiftllm_b200.sampling.batch import row_keys
    seed = np.array([-1, 5, 2 ** 40 + 3, -1, 0])
    si = np.array([3, 7, 9, 2 ** 33 + 1, 0])
    k, c0, c1 = row_keys(seed, si, 1234, 77)
    for i in range(5):
        if seed[i] >= 0:
            assert (k[i], c0[i], c1[i]) == (mix_key(int(seed[i]), 0x5EED), int(si[i]) & 0xFFFFFFFF, 0)
        else:
            assert (k[i], c0[i], c1[i]) == (mix_key(1234, 0xA11), 77, i)
