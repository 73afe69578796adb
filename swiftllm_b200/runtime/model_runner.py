"""Per-rank model runner: weights, the paged KV pool, step execution and
CUDA-graph replay for decode steps.

Parity: crates/swiftllm-core/src/execution/mod.rs (ModelExecutor trait
:18-43, BatchBuilder :46-126, ExecutionStats :128-193, CudaGraphCache keyed
by batch size :230-284) and crates/swiftllm-core/src/memory/{mod.rs,
kv_cache.rs} (MemoryPool sizing, KV geometry). The reference sizes the pool
from a hard-coded 16 GB (engine.rs:66-80); here it comes from a profiling
forward pass and ``torch.cuda.mem_get_info``.

KV pool layout: one tensor [num_blocks, num_layers, 2, kv_heads, block_size,
head_dim]. A block's data for every layer is contiguous, so a copy-on-write
or a swap of one block is a single contiguous copy, and one (block, layer,
k|v, head) page is a contiguous block_size x head_dim tile for the attention
kernels.
"""

from __future__ import annotations

import math
import os
import time
from dataclasses import dataclass
from typing import Dict, List, Optional, Tuple

import numpy as np
import torch

from .. import ops
from ..models.config import ModelConfig
from ..models.decoder import AttnMeta, DecoderModel, TPGroup
from ..utils.logging import get_logger
from ..utils import nvtx

log = get_logger(__name__)

_GRAPH_BATCHES = [1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256,
                  320, 384, 448, 512]


@dataclass
class StepInput:
    """Host-side view of one scheduled step (what rank 0 broadcasts)."""
    num_seqs: int
    num_decode_seqs: int
    num_tokens: int
    max_q_len: int
    max_seq_len: int
    max_blocks: int
    ints: np.ndarray          # packed int32 (see Batch.pack_int32)
    logits_idx: np.ndarray    # int32 flat token rows whose logits are needed
    swap_in: np.ndarray       # [n, 2] (cpu, gpu)
    swap_out: np.ndarray      # [n, 2] (gpu, cpu)
    copies: np.ndarray        # [n, 2] (src, dst)
    greedy: bool = False      # every sampled row is greedy, no logprobs / penalties


@dataclass
class GreedyResult:
    """Device tensors [len(logits_idx)]: argmax token over the full
    vocabulary and its log-probability (vocab-parallel greedy sampling)."""
    tokens: torch.Tensor
    lps: torch.Tensor


def step_input_from_batch(b) -> StepInput:
    q_start = np.asarray(b.q_start)
    q_len = np.asarray(b.q_len)
    last = (q_start[:-1] + q_len - 1).astype(np.int32)
    # rows that sample: unique logits rows in order (sample_logit_idx indexes this list)
    seq_rows = np.asarray(b.sample_seq_row)
    lrows = np.asarray(b.sample_logit_idx)
    n_logits = int(lrows.max()) + 1 if lrows.size else 0
    logits_idx = np.zeros(n_logits, dtype=np.int32)
    if lrows.size:
        logits_idx[lrows] = last[seq_rows]
    return StepInput(b.num_seqs, b.num_decode_seqs, int(b.num_tokens), b.max_q_len,
                     b.max_seq_len, b.max_blocks, b.pack_int32(), logits_idx,
                     b.swap_in, b.swap_out, b.copies)


def prefill_step_input(ids, block_size: int, n_logits: int = 1) -> StepInput:
    """A one-sequence prefill step over KV blocks 0.. (for checks run on a
    fresh pool, before any request owns a block): logits of the last
    ``n_logits`` positions."""
    T = len(ids)
    nb = (T + block_size - 1) // block_size
    ints = np.concatenate([np.asarray(ids, dtype=np.int32), np.arange(T, dtype=np.int32),
                           np.arange(T, dtype=np.int32), np.array([0, T], dtype=np.int32),
                           np.array([T], dtype=np.int32), np.arange(nb, dtype=np.int32)])
    empty = np.zeros((0, 2), dtype=np.int64)
    return StepInput(1, 0, T, T, T, nb, ints,
                     np.arange(T - n_logits, T, dtype=np.int32), empty, empty, empty)


class ModelRunner:
    def __init__(self, model_cfg: ModelConfig, engine_cfg, device: torch.device,
                 tp: Optional[TPGroup] = None, max_model_len: Optional[int] = None):
        self.cfg = model_cfg
        self.ecfg = engine_cfg
        self.device = torch.device(device)
        self.is_cuda = self.device.type == "cuda"
        self.tp = tp or TPGroup()
        self.dtype = self._resolve_dtype(engine_cfg.dtype)
        self.max_model_len = max_model_len or min(model_cfg.max_position_embeddings, 4096)
        self.block_size = engine_cfg.block_size
        self.model = DecoderModel(model_cfg, self.dtype, self.device, self.tp,
                                  max_pos=max(self.max_model_len, 1) + 1)
        self.kv_cache: Optional[torch.Tensor] = None
        self.cpu_cache: Optional[torch.Tensor] = None
        self.num_gpu_blocks = 0
        self.num_cpu_blocks = 0
        self.graphs: Dict[int, Tuple[torch.cuda.CUDAGraph, dict]] = {}
        self.graph_pool = None
        self.use_graphs = (self.is_cuda and engine_cfg.enable_cuda_graphs
                           and not engine_cfg.enforce_eager)
        self.max_blocks_per_seq = (self.max_model_len + self.block_size - 1) // self.block_size
        self.stats = {"steps": 0, "graph_steps": 0, "tokens": 0}
        self._decode_ws = None

    def _resolve_dtype(self, dt) -> torch.dtype:
        v = getattr(dt, "value", dt)
        if v == "float32":
            return torch.float32
        if v == "float16":
            return torch.float16
        if v == "bfloat16":
            return torch.bfloat16
        return torch.bfloat16 if self.is_cuda else torch.float32

    # ----------------------------------------------------------- weights
    def load_weights(self) -> None:
        t0 = time.time()
        self.model.allocate()
        fmt = self.ecfg.load_format
        model = self.ecfg.model
        q = getattr(self.ecfg.quantization, "value", self.ecfg.quantization)
        group = 128
        if fmt == "dummy" or (fmt == "auto" and not os.path.exists(model)):
            self.model.init_dummy(seed=self.ecfg.seed)
        else:
            from ..loaders import open_checkpoint
            from ..loaders.quantized import wrap_quantized
            ckpt = open_checkpoint(model, fmt)
            get, found = wrap_quantized(ckpt.get, model)
            if found is not None:  # GPTQ / AWQ tensors: dequantised here, re-packed below
                group = found[1]
                if q in (None, "none"):
                    q = "int4"
            self.model.load_state(get)
        if q == "fp8":
            self.model.quantize_fp8()
        elif q == "int8":
            self.model.quantize_int8()
        elif q in ("int4", "gptq", "awq"):
            self.model.quantize_int4(group)
        elif q == "nvfp4":
            self.model.quantize_nvfp4()
        elif q not in (None, "none"):
            raise NotImplementedError(f"quantization {q!r} is not supported "
                                      "(fp8, int8, int4 / gptq / awq, nvfp4 are)")
        elif (self.is_cuda and ops.gemm_backend() == "tcgen05"
              and os.environ.get("SWIFTLLM_FUSE_SWIGLU", "1") != "0"):
            # our GEMMs everywhere: SwiGLU in the gate/up GEMM epilogue
            # ("auto" runs the library gate/up GEMM and our SiLU-mul kernel:
            # measured faster at every token count)
            self.model.fuse_swiglu()
        if self.is_cuda:
            self.model.pad_k()
            torch.cuda.synchronize(self.device)
        log.info("weights ready in %.1fs (%s, rank %d/%d)", time.time() - t0, fmt,
                 self.tp.rank, self.tp.size)

    # ----------------------------------------------------------- KV pool
    def block_bytes(self) -> int:
        c = self.cfg
        el = torch.tensor([], dtype=self.dtype).element_size()
        return c.num_layers * 2 * self.model.local_kv_heads * self.block_size * c.head_dim * el

    def profile_num_blocks(self) -> int:
        if self.ecfg.num_gpu_blocks_override:
            return int(self.ecfg.num_gpu_blocks_override)
        if not self.is_cuda:
            budget = int(os.environ.get("SWIFTLLM_CPU_KV_BYTES", 256 << 20))
            return max(16, budget // self.block_bytes())
        torch.cuda.synchronize(self.device)
        torch.cuda.empty_cache()
        torch.cuda.reset_peak_memory_stats(self.device)
        # profiling pass: the largest prefill a step may run, with a tiny KV pool
        n_tok = min(self.ecfg.max_num_batched_tokens or 8192, 16384)
        self.allocate_kv(max(4, (n_tok + self.block_size - 1) // self.block_size + 1), 0)
        ids = torch.zeros(n_tok, dtype=torch.int32, device=self.device)
        nb = (n_tok + self.block_size - 1) // self.block_size
        meta = AttnMeta(
            num_seqs=1, num_decode_seqs=0, num_tokens=n_tok, max_q_len=n_tok, max_seq_len=n_tok,
            positions=torch.arange(n_tok, dtype=torch.int32, device=self.device) % self.max_model_len,
            slot_mapping=torch.arange(n_tok, dtype=torch.int32, device=self.device),
            q_start=torch.tensor([0, n_tok], dtype=torch.int32, device=self.device),
            seq_lens=torch.tensor([n_tok], dtype=torch.int32, device=self.device),
            block_tables=torch.arange(nb, dtype=torch.int32, device=self.device).view(1, nb),
            logits_idx=torch.arange(min(n_tok, self.ecfg.max_num_seqs), dtype=torch.int32,
                                    device=self.device))
        h = self.model.forward(ids, meta, self.kv_cache)
        self.model.compute_logits(h)
        torch.cuda.synchronize(self.device)
        peak = torch.cuda.max_memory_allocated(self.device)
        kv_now = self.kv_cache.numel() * self.kv_cache.element_size()
        self.kv_cache = None
        torch.cuda.empty_cache()
        free, total = torch.cuda.mem_get_info(self.device)
        used_by_others = total - free - torch.cuda.memory_reserved(self.device)
        budget = total * self.ecfg.gpu_memory_utilization - (peak - kv_now) - max(used_by_others, 0)
        budget -= 2 << 30  # graphs, sampler scratch, NCCL / comm buffers
        # a speculative draft model keeps its weights and one KV block per
        # target block on the same GPU
        budget -= getattr(self.ecfg, "draft_reserve_bytes", 0)
        n = int(budget // (self.block_bytes() + getattr(self.ecfg, "draft_block_bytes", 0)))
        if n <= 0:
            raise RuntimeError("no GPU memory left for the KV cache; lower max_num_batched_tokens "
                               "or raise gpu_memory_utilization")
        return n

    def allocate_kv(self, num_gpu_blocks: int, num_cpu_blocks: int) -> None:
        c = self.cfg
        shape = (num_gpu_blocks, c.num_layers, 2, self.model.local_kv_heads, self.block_size,
                 c.head_dim)
        self.kv_cache = torch.zeros(shape, dtype=self.dtype, device=self.device)
        self.num_gpu_blocks = num_gpu_blocks
        if num_cpu_blocks > 0:
            cshape = (num_cpu_blocks,) + shape[1:]
            self.cpu_cache = torch.zeros(cshape, dtype=self.dtype,
                                         pin_memory=self.is_cuda)
        self.num_cpu_blocks = num_cpu_blocks

    def num_cpu_blocks_for(self, swap_gib: float) -> int:
        return int(swap_gib * (1 << 30) // self.block_bytes())

    # ----------------------------------------------------------- step
    def _decode_splits(self, num_decode: int, max_seq_len: int) -> int:
        # split-KV so that decode fills the GPU (148 SMs) when the batch is small
        if num_decode == 0:
            return 1
        heads = self.model.local_kv_heads
        want = max(1, (2 * 148) // max(1, num_decode * heads))
        chunks = max(1, (max_seq_len + 255) // 256)
        return int(min(want, chunks, 32))

    def _workspace(self, rows: int, splits: int) -> torch.Tensor:
        # partial outputs + (max, sum) per (row, head, split)
        need = rows * self.model.local_heads * splits * (self.cfg.head_dim + 2)
        if self._decode_ws is None or self._decode_ws.numel() < need:
            self._decode_ws = torch.empty(max(need, 1 << 20), dtype=torch.float32, device=self.device)
        return self._decode_ws

    def _meta_from(self, si: StepInput, ints: torch.Tensor, logits_idx: torch.Tensor) -> Tuple[torch.Tensor, AttnMeta]:
        T, S, MB = si.num_tokens, si.num_seqs, si.max_blocks
        o = 0
        input_ids = ints[o:o + T]; o += T
        positions = ints[o:o + T]; o += T
        slots = ints[o:o + T]; o += T
        q_start = ints[o:o + S + 1]; o += S + 1
        seq_lens = ints[o:o + S]; o += S
        bt = ints[o:o + S * MB].view(S, MB)
        splits = self._decode_splits(si.num_decode_seqs, si.max_seq_len) if self.is_cuda else 1
        meta = AttnMeta(num_seqs=S, num_decode_seqs=si.num_decode_seqs, num_tokens=T,
                        max_q_len=si.max_q_len, max_seq_len=si.max_seq_len, positions=positions,
                        slot_mapping=slots, q_start=q_start, seq_lens=seq_lens, block_tables=bt,
                        logits_idx=logits_idx, decode_splits=splits,
                        decode_workspace=self._workspace(max(si.num_decode_seqs, 1), splits)
                        if self.is_cuda else None)
        return input_ids, meta

    def _apply_cache_ops(self, si: StepInput) -> None:
        if si.swap_out.size:
            self.swap(si.swap_out, to_host=True)
        if si.swap_in.size:
            self.swap(si.swap_in, to_host=False)
        if si.copies.size:
            ops.copy_blocks(self.kv_cache, torch.from_numpy(si.copies).to(self.device))

    def swap(self, pairs: np.ndarray, to_host: bool) -> None:
        """Block swap between the GPU pool and the pinned host pool, one
        contiguous copy per block (all layers)."""
        if self.cpu_cache is None:
            raise RuntimeError("swap requested but no host swap space is allocated")
        for a, b in pairs.tolist():
            if to_host:
                self.cpu_cache[b].copy_(self.kv_cache[a], non_blocking=True)
            else:
                self.kv_cache[b].copy_(self.cpu_cache[a], non_blocking=True)
        if self.is_cuda and to_host:
            torch.cuda.current_stream(self.device).synchronize()

    @torch.inference_mode()
    def execute(self, si: StepInput) -> Optional[torch.Tensor]:
        """Runs one step; returns fp32 logits [len(logits_idx), vocab] (all ranks)."""
        self.stats["steps"] += 1
        self.stats["tokens"] += si.num_tokens
        self._apply_cache_ops(si)
        if si.num_tokens == 0:
            return None
        with nvtx.range("prepare"):
            if self.is_cuda:
                ints = torch.from_numpy(si.ints).pin_memory().to(self.device, non_blocking=True)
                lidx = torch.from_numpy(si.logits_idx).pin_memory().to(self.device, non_blocking=True)
            else:
                ints = torch.from_numpy(si.ints)
                lidx = torch.from_numpy(si.logits_idx)
        pure_decode = si.num_decode_seqs == si.num_seqs and si.logits_idx.size == si.num_seqs
        if self.use_graphs and pure_decode and self.graphs:
            g = self._graph_for(si.num_seqs)
            if g is not None:
                return self._replay(g, si, ints)
        input_ids, meta = self._meta_from(si, ints, lidx)
        with nvtx.range("forward"):
            h = self.model.forward(input_ids, meta, self.kv_cache)
            return self._finish_logits(self.model.compute_logits(h, gather=False), si)

    def _finish_logits(self, local: torch.Tensor, si: StepInput):
        """Full-vocabulary fp32 logits, or, for an all-greedy step under
        vocab-parallel TP with the fused backend, the merged greedy result
        (no logits gather). Every rank calls this with the same ``si``."""
        if not self.model.vocab_parallel:
            return local
        if si.greedy and hasattr(self.tp, "vocab_greedy"):
            tok, lp = self.tp.vocab_greedy(local, self.model.vocab_start)
            return GreedyResult(tok, lp)
        return self.tp.gather_vocab(local)

    def release(self) -> None:
        """Drop the graphs, the KV pools and the weights so their device
        memory can be reused in the same process (bench arms run back to
        back); the runner is unusable afterwards."""
        if self.is_cuda:
            torch.cuda.synchronize(self.device)
        self.graphs = {}
        self._gbuf = None
        self.graph_pool = None
        self.kv_cache = None
        self.cpu_cache = None
        self._decode_ws = None
        self.model = None
        close = getattr(self.tp, "close", None)
        if close is not None:
            close()
        if self.is_cuda:
            import gc
            gc.collect()
            torch.cuda.empty_cache()

    # ----------------------------------------------------------- CUDA graphs
    def _graph_for(self, n: int) -> Optional[int]:
        for b in sorted(self.graphs):
            if b >= n:
                return b
        return None

    @torch.inference_mode()
    def capture_graphs(self, max_batch: int) -> None:
        if not self.use_graphs:
            return
        t0 = time.time()
        dev = self.device
        MB = self.max_blocks_per_seq
        sizes = [b for b in _GRAPH_BATCHES if b <= max_batch]
        if not sizes or sizes[-1] < max_batch:
            sizes.append(max_batch)
        bmax = sizes[-1]
        self._gbuf = {
            "ids": torch.zeros(bmax, dtype=torch.int32, device=dev),
            "pos": torch.zeros(bmax, dtype=torch.int32, device=dev),
            "slots": torch.full((bmax,), -1, dtype=torch.int32, device=dev),
            "q_start": torch.arange(bmax + 1, dtype=torch.int32, device=dev),
            "seq_lens": torch.zeros(bmax, dtype=torch.int32, device=dev),
            "bt": torch.zeros(bmax, MB, dtype=torch.int32, device=dev),
            "lidx": torch.arange(bmax, dtype=torch.int32, device=dev),
        }
        self.graph_pool = torch.cuda.graph_pool_handle()
        for b in reversed(sizes):
            splits = self._decode_splits(b, self.max_model_len)
            ws = self._workspace(b, splits)
            buf = self._gbuf
            meta = AttnMeta(num_seqs=b, num_decode_seqs=b, num_tokens=b, max_q_len=1,
                            max_seq_len=self.max_model_len, positions=buf["pos"][:b],
                            slot_mapping=buf["slots"][:b], q_start=buf["q_start"][:b + 1],
                            seq_lens=buf["seq_lens"][:b], block_tables=buf["bt"][:b],
                            logits_idx=buf["lidx"][:b], decode_splits=splits,
                            decode_workspace=ws)
            # warm up outside capture (allocator, lazy init)
            s = torch.cuda.Stream(dev)
            s.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(s):
                for _ in range(2):
                    h = self.model.forward(buf["ids"][:b], meta, self.kv_cache)
                    self.model.compute_logits(h, gather=False)
            torch.cuda.current_stream(dev).wait_stream(s)
            g = torch.cuda.CUDAGraph()
            n0 = ops.LAUNCHES[0]
            with torch.cuda.graph(g, pool=self.graph_pool):
                h = self.model.forward(buf["ids"][:b], meta, self.kv_cache)
                out = self.model.compute_logits(h, gather=False)
            self.graphs[b] = (g, {"out": out, "launches": ops.LAUNCHES[0] - n0})
            ops.LAUNCHES[0] = n0
        torch.cuda.synchronize(dev)
        log.info("captured %d decode graphs (max batch %d) in %.1fs", len(self.graphs), bmax,
                 time.time() - t0)

    def _replay(self, b: int, si: StepInput, ints: torch.Tensor) -> torch.Tensor:
        g, io = self.graphs[b]
        n = si.num_seqs
        MB = si.max_blocks
        buf = self._gbuf
        o = 0
        buf["ids"][:n].copy_(ints[o:o + n]); o += n
        buf["pos"][:n].copy_(ints[o:o + n]); o += n
        buf["slots"][:n].copy_(ints[o:o + n]); o += n
        o += n + 1  # q_start: static arange
        buf["seq_lens"][:n].copy_(ints[o:o + n]); o += n
        if n < b:
            buf["slots"][n:b].fill_(-1)
            buf["seq_lens"][n:b].fill_(0)
        buf["bt"][:n, :MB].copy_(ints[o:o + n * MB].view(n, MB))
        g.replay()
        ops.LAUNCHES[0] += io["launches"]
        self.stats["graph_steps"] += 1
        return self._finish_logits(io["out"][:n], si)
