"""Executors: run a step on every tensor-parallel rank.

* ``LocalExecutor``: this process owns rank 0's runner. For tp > 1 the other
  ranks are either spawned here (one process per GPU, ``LLM(tensor_parallel_
  size=k)``) or already running the same program under torchrun (``bench.py``),
  in which case they sit in :func:`worker_loop`.
* Step metadata travels rank 0 -> workers over the shared-memory channel
  (csrc/core/shm_channel.cpp); the tensors never leave the GPUs except the
  all-reduces / fused reductions inside the forward.

Parity: crates/swiftllm-core/src/execution/tensor_parallel.rs
(TensorParallelExecutor :66-203; broadcast / barrier stubs :144-159).
"""

from __future__ import annotations

import os
import pickle
import threading
import time
import uuid
from typing import Optional

import numpy as np
import torch

from .. import _core
from ..utils.logging import get_logger
from .comm import build_tp_group, init_distributed

log = get_logger(__name__)

_SHUTDOWN = b"__shutdown__"
STEP_TIMEOUT = float(os.environ.get("SWIFTLLM_STEP_TIMEOUT", "600"))
# a worker whose heartbeat is older than this is reported dead; workers
# likewise give up on an engine whose heartbeat stopped
PEER_TIMEOUT = float(os.environ.get("SWIFTLLM_PEER_TIMEOUT", "60"))
HEARTBEAT_PERIOD = 0.5


def _device_for(cfg, local_rank: int) -> torch.device:
    want = cfg.device
    if want == "cpu" or (want == "auto" and not torch.cuda.is_available()):
        return torch.device("cpu")
    torch.cuda.set_device(local_rank)
    return torch.device("cuda", local_rank)


def _build_runner(model_cfg, cfg, rank: int, world: int, local_rank: int):
    from ..runtime.model_runner import ModelRunner
    device = _device_for(cfg, local_rank)
    tp = build_tp_group(rank, world, device, cfg.comm_backend, model_cfg,
                        max(int(cfg.max_num_batched_tokens or 8192), 16384))
    if device.type == "cuda":
        # the NCCL backend is the library baseline: cuBLAS GEMMs + NCCL
        # all-reduce; otherwise the process default ("auto" unless
        # SWIFTLLM_GEMM says otherwise)
        from .. import ops
        ops.set_gemm_backend("cublas" if cfg.comm_backend == "nccl" else ops.DEFAULT_GEMM_BACKEND)
    runner = ModelRunner(model_cfg, cfg, device, tp, cfg.max_model_len)
    runner.load_weights()
    n = runner.profile_num_blocks()
    if world > 1:
        import torch.distributed as dist
        t = torch.tensor([n], dtype=torch.int64, device=device if device.type == "cuda" else "cpu")
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        n = int(t.item())
    n_cpu = runner.num_cpu_blocks_for(cfg.swap_space) if cfg.preemption_mode.value == "swap" else 0
    if device.type == "cpu":
        n_cpu = min(n_cpu, 64)
    runner.allocate_kv(n, n_cpu)
    runner.capture_graphs(cfg.max_num_seqs)
    return runner


def worker_loop(model_cfg, cfg, rank: int, world: int, local_rank: int, channel_name: str) -> None:
    """Body of a tensor-parallel worker rank: build the runner, then execute
    every step rank 0 publishes until shutdown."""
    runner = _build_runner(model_cfg, cfg, rank, world, local_rank)
    ch = None
    for _ in range(2000):
        try:
            ch = _core.ShmChannel(channel_name, False, world - 1, rank - 1)
            break
        except RuntimeError:
            time.sleep(0.01)
    if ch is None:
        raise RuntimeError("worker could not attach to the control channel")
    while True:
        try:
            msg = ch.receive(timeout=-1.0, peer_timeout=PEER_TIMEOUT)
        except _core.PeerDiedError as e:
            log.error("rank %d: %s; exiting", rank, e)
            raise SystemExit(3)
        if msg == _SHUTDOWN:
            break
        obj = pickle.loads(msg)
        if isinstance(obj, tuple):  # control message: ("timer", "start" | "stop" | "report")
            _timer_op(runner, obj[1])
            continue
        runner.execute(obj)
    del ch
    runner.release()


def run_worker_from_env(cfg) -> None:
    """Entry for ranks != 0 of a torchrun job (bench.py): join the process
    group, build this rank's runner and serve rank 0's steps until shutdown.
    Returns after rank 0's shutdown with this rank's device memory released
    (the process group stays up for a later engine or the final teardown)."""
    from ..engine.llm_engine import prepare_config
    model_cfg = prepare_config(cfg)
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local_rank = int(os.environ.get("LOCAL_RANK", rank))
    backend = "nccl" if cfg.device != "cpu" and torch.cuda.is_available() else "gloo"
    init_distributed(rank, world, backend)
    cname = os.environ.get("SWIFTLLM_CHANNEL", "/swiftllm-torchrun-" + os.environ.get("MASTER_PORT", "0"))
    worker_loop(model_cfg, cfg, rank, world, local_rank, cname)


class _Timer:
    def __init__(self):
        self.start = self.end = None
        self.t0 = 0.0
        self.ms = 0.0


_TIMER = _Timer()


def _timer_op(runner, op: str) -> float:
    """Timed window over engine steps on every rank: barrier + synchronize on
    both sides, CUDA events on the launching stream, max over ranks."""
    import torch.distributed as dist
    dev = runner.device
    multi = dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1
    if op == "start":
        if runner.is_cuda:
            torch.cuda.synchronize(dev)
        if multi:
            dist.barrier()
        if runner.is_cuda:
            torch.cuda.synchronize(dev)
            _TIMER.start = torch.cuda.Event(enable_timing=True)
            _TIMER.end = torch.cuda.Event(enable_timing=True)
            _TIMER.start.record()
        else:
            _TIMER.t0 = time.perf_counter()
        return 0.0
    if op == "stop":
        if runner.is_cuda:
            _TIMER.end.record()
            torch.cuda.synchronize(dev)
            _TIMER.ms = _TIMER.start.elapsed_time(_TIMER.end)
        else:
            _TIMER.ms = (time.perf_counter() - _TIMER.t0) * 1e3
        if multi:
            dist.barrier()
        return _TIMER.ms
    if op == "report":
        v = _TIMER.ms
        if multi:
            t = torch.tensor([v], dtype=torch.float64, device=dev if runner.is_cuda else "cpu")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            v = float(t.item())
        return v
    raise ValueError(op)


def _spawn_entry(rank, model_cfg, cfg, world, channel_name, port):
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port),
                       "RANK": str(rank), "WORLD_SIZE": str(world), "LOCAL_RANK": str(rank)})
    init_distributed(rank, world, "nccl" if cfg.device != "cpu" and torch.cuda.is_available() else "gloo")
    worker_loop(model_cfg, cfg, rank, world, rank, channel_name)


class LocalExecutor:
    def __init__(self, model_cfg, cfg):
        self.cfg = cfg
        world = cfg.tensor_parallel_size
        self.world = world
        self.procs = []
        self.channel = None
        env_world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        if world > 1:
            cname = os.environ.get("SWIFTLLM_CHANNEL") or f"/swiftllm-{os.getpid()}-{uuid.uuid4().hex[:8]}"
            if env_world == world:
                # launched by torchrun: workers are the other ranks of this job
                init_distributed(rank, world, self._backend())
                if rank != 0:
                    raise RuntimeError("LocalExecutor must live on rank 0; call worker_loop elsewhere")
                cname = os.environ.get("SWIFTLLM_CHANNEL", "/swiftllm-torchrun-" + os.environ.get("MASTER_PORT", "0"))
            else:
                import torch.multiprocessing as mp
                port = _free_port()
                ctx = mp.get_context("spawn")
                for r in range(1, world):
                    p = ctx.Process(target=_spawn_entry, args=(r, model_cfg, cfg, world, cname, port),
                                    daemon=True)
                    p.start()
                    self.procs.append(p)
                os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
                init_distributed(0, world, self._backend())
            self.channel = _core.ShmChannel(cname, True, world - 1, -1, 8, 16 << 20)
            self._beat_stop = threading.Event()
            self._beat = threading.Thread(target=self._beat_loop, name="swiftllm-heartbeat",
                                          daemon=True)
            self._beat.start()
        self.runner = _build_runner(model_cfg, cfg, 0, world, local_rank if env_world == world else 0)
        self.device = self.runner.device
        self.num_gpu_blocks = self.runner.num_gpu_blocks
        self.num_cpu_blocks = self.runner.num_cpu_blocks

    def _backend(self) -> str:
        return "nccl" if self.cfg.device != "cpu" and torch.cuda.is_available() else "gloo"

    def timer(self, op: str) -> float:
        """Start / stop / report the device-timed window on every rank."""
        if self.channel is not None:
            self.channel.publish(pickle.dumps(("timer", op)), STEP_TIMEOUT)
        return _timer_op(self.runner, op)

    def execute(self, si):
        if self.channel is not None:
            self._check_workers()
            self.channel.publish(pickle.dumps(si, protocol=pickle.HIGHEST_PROTOCOL), STEP_TIMEOUT)
        return self.runner.execute(si)

    def _beat_loop(self) -> None:
        # the engine's heartbeat: workers waiting for a step see it advance
        # even when no request arrives for a long time
        ch = self.channel
        while not self._beat_stop.wait(HEARTBEAT_PERIOD):
            if ch is None or ch.closed:
                break
            ch.beat()

    def _check_workers(self) -> None:
        from .failures import WorkerDiedError
        for p in self.procs:
            if not p.is_alive():
                raise WorkerDiedError(f"tensor-parallel worker pid {p.pid} exited "
                                      f"(code {p.exitcode})")
        for r in range(1, self.world):
            age = self.channel.heartbeat_age(r)
            # age < 0: the worker has not attached yet (still loading)
            if age > PEER_TIMEOUT:
                raise WorkerDiedError(f"tensor-parallel rank {r} heartbeat lost "
                                      f"({age:.1f} s old)")

    def shutdown(self) -> None:
        if self.channel is not None:
            self._beat_stop.set()
            try:
                self.channel.publish(_SHUTDOWN, 5.0)
            except Exception:
                pass
            for p in self.procs:
                p.join(timeout=10)
                if p.is_alive():
                    p.terminate()
            self.channel.close()
            self.channel = None
        if self.runner is not None:
            self.runner.release()
            self.runner = None


def _free_port() -> int:
    import socket
    with socket.socket(socket.AF_INET, socket.SOCK_STREAM) as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_executor(model_cfg, cfg) -> LocalExecutor:
    return LocalExecutor(model_cfg, cfg)
