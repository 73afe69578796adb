"""Failure detection on the host (no GPU, no device fault): the control
channel's bounded waits and heartbeats, and the engine noticing a dead
tensor-parallel worker (a gloo rank killed between steps)."""

import os
import signal
import time
import uuid

import pytest

from swiftllm_b200 import LLM, SamplingParams, _core
from swiftllm_b200.parallel.failures import WorkerDiedError, is_timeout


def _name():
    return f"/swt-{os.getpid()}-{uuid.uuid4().hex[:6]}"


def test_channel_timeouts_and_heartbeats():
    name = _name()
    w = _core.ShmChannel(name, True, 1, -1, 2, 1024)
    r = _core.ShmChannel(name, False, 1, 0)
    # no message: the reader's bounded wait ends with a timeout error
    t0 = time.time()
    with pytest.raises(_core.ChannelTimeoutError) as ei:
        r.receive(timeout=0.2)
    assert is_timeout(ei.value) and time.time() - t0 < 5
    w.publish(b"step-1", 1.0)
    assert r.receive(timeout=1.0) == b"step-1"
    # a reader that stops reading: the ring fills, then publish times out
    w.publish(b"a", 1.0)
    w.publish(b"b", 1.0)
    with pytest.raises(_core.ChannelTimeoutError):
        w.publish(b"c", 0.2)
    assert r.receive(timeout=1.0) == b"a" and r.receive(timeout=1.0) == b"b"
    # the engine's heartbeat goes stale: the reader reports a dead peer
    time.sleep(0.4)
    with pytest.raises(_core.PeerDiedError):
        r.receive(timeout=5.0, peer_timeout=0.3)
    # a fresh beat keeps the reader waiting (it times out instead)
    w.beat()
    with pytest.raises(_core.ChannelTimeoutError):
        r.receive(timeout=0.1, peer_timeout=5.0)
    # closing wakes the reader with a dead-peer error
    w.close()
    with pytest.raises(_core.PeerDiedError):
        r.receive(timeout=5.0)
    # the reader's own heartbeat is visible to the writer
    assert w.heartbeat_age(1) < 5.0


def test_dead_tp_worker_is_reported():
    llm = LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32",
              tensor_parallel_size=2, max_model_len=128)
    sp = SamplingParams(temperature=0, max_tokens=4, ignore_eos=True)
    out = llm.generate(prompt_token_ids=[[1, 2, 3, 4]], sampling_params=sp, use_tqdm=False)
    assert len(out[0].outputs[0].token_ids) == 4
    ex = llm.llm_engine.executor
    assert len(ex.procs) == 1
    pid = ex.procs[0].pid
    os.kill(pid, signal.SIGKILL)  # the worker this test spawned, by exact pid
    ex.procs[0].join(timeout=30)
    # the step that finds the dead worker finishes the in-flight request as aborted
    out = llm.generate(prompt_token_ids=[[5, 6, 7]], sampling_params=sp, use_tqdm=False)
    assert out[0].outputs[0].finish_reason.value == "abort"
    # and the engine refuses further work with the original error
    with pytest.raises(WorkerDiedError):
        llm.generate(prompt_token_ids=[[8, 9]], sampling_params=sp, use_tqdm=False)
    llm.shutdown()


def test_request_timeout_aborts():
    llm = LLM("tiny-llama", load_format="dummy", device="cpu", dtype="float32",
              max_model_len=128, request_timeout_secs=0.05)
    eng = llm.llm_engine
    sp = SamplingParams(temperature=0, max_tokens=100, ignore_eos=True)
    eng.add_request("slow", prompt_token_ids=[1, 2, 3], sampling_params=sp)
    outs = []
    t0 = time.time()
    while eng.has_unfinished_requests() and time.time() - t0 < 60:
        outs += eng.step()
        time.sleep(0.01)
    fin = [o for o in outs if o.finished]
    assert fin and fin[0].outputs[0].finish_reason.value == "abort"
    assert len(fin[0].outputs[0].token_ids) < 100
