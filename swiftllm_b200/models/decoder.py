"""Decoder-only transformer covering the Llama family (Llama 2/3, Mistral,
Qwen2 with qkv bias), Mixtral (MoE) and Phi (LayerNorm, GELU, partial
rotary, parallel attention/MLP block).

Parity: crates/swiftllm-models/src/architectures/{llama.rs, mistral.rs,
qwen.rs, phi.rs} (structure only in the reference: its forward returns zeros)
and crates/swiftllm-models/src/layers/* (QKVProjection :152-192,
GateUpProjection :194-224, FusedGatedMlp mlp.rs:169-205, MoeMlp
mlp.rs:207-258, FusedAddRMSNorm normalization.rs:153-180).

Layout (one process per GPU, tensor parallel over ``tp.size`` ranks):
  wqkv   [(Hq + 2 Hkv) D / tp, H]  column-parallel, q heads then k then v
  wo     [H, Hq D / tp]            row-parallel -> reduction across ranks
  w13    [2 I / tp, H]             gate rows then up rows (per rank)
  w2     [H, I / tp]               row-parallel -> reduction across ranks
  MoE    router [E, H] (replicated), w13 [E, 2 I / tp, H], w2 [E, H, I / tp]
Under the fused backend the residual stream is sharded by token rows and
each row-parallel reduction is one kernel that also adds the residual,
normalises and all-gathers (``_forward_seq_parallel``, ``tp.reduce_norm``);
under the NCCL baseline the residual is replicated and each row-parallel
output is all-reduced (``tp.reduce``).
"""

from __future__ import annotations

import math
import zlib
from dataclasses import dataclass
from types import SimpleNamespace
from typing import Callable, Dict, List, Optional

import torch

from .. import ops
from .config import ModelConfig
from .rope import cos_sin_table


@dataclass
class AttnMeta:
    """Device-side metadata of one step (see csrc/core/scheduler.h Batch)."""
    num_seqs: int
    num_decode_seqs: int
    num_tokens: int
    max_q_len: int
    max_seq_len: int
    positions: torch.Tensor
    slot_mapping: torch.Tensor
    q_start: torch.Tensor
    seq_lens: torch.Tensor
    block_tables: torch.Tensor
    logits_idx: torch.Tensor
    decode_splits: int = 1
    decode_workspace: Optional[torch.Tensor] = None


class TPGroup:
    """Tensor-parallel group handle used by the model. Single-rank default."""

    def __init__(self, rank: int = 0, size: int = 1):
        self.rank = rank
        self.size = size

    def reduce(self, x: torch.Tensor) -> torch.Tensor:
        """Sum partial activations across ranks (row-parallel output)."""
        return x

    def gather_vocab(self, x: torch.Tensor) -> torch.Tensor:
        """Concatenate vocab-parallel logits along the last dim."""
        return x

    def linear_reduce(self, x: torch.Tensor, w: torch.Tensor,
                      b: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Row-parallel linear followed by the cross-rank sum (the bias, if
        any, is added once)."""
        if self.size > 1 and self.rank != 0:
            b = None
        return self.reduce(ops.linear(x, w, b))


def _shard(n: int, rank: int, size: int):
    if n % size:
        raise ValueError(f"dimension {n} not divisible by tensor-parallel size {size}")
    s = n // size
    return rank * s, (rank + 1) * s


def tensor_id(name: str) -> int:
    return zlib.crc32(name.encode()) & 0x7FFFFFFF


class DecoderModel:
    def __init__(self, cfg: ModelConfig, dtype: torch.dtype, device: torch.device,
                 tp: Optional[TPGroup] = None, max_pos: Optional[int] = None):
        self.cfg = cfg
        self.dtype = dtype
        self.device = torch.device(device)
        self.tp = tp or TPGroup()
        r, n = self.tp.rank, self.tp.size
        if cfg.num_heads % n:
            raise ValueError("num_heads must be divisible by tensor_parallel_size")
        self.local_heads = cfg.num_heads // n
        # KV heads: split when possible, else replicate (MQA / small GQA)
        if cfg.num_kv_heads % n == 0:
            self.local_kv_heads = cfg.num_kv_heads // n
            self.kv_head_start = r * self.local_kv_heads
        else:
            if n % cfg.num_kv_heads:
                raise ValueError("kv heads must divide or be divisible by tensor_parallel_size")
            self.local_kv_heads = 1
            self.kv_head_start = r * cfg.num_kv_heads // n
        self.local_inter = cfg.intermediate_size // n
        # MoE: expert parallel when the experts divide over the ranks (each rank
        # keeps E/n whole experts), else every rank keeps an I/n slice of all
        self.ep = bool(cfg.num_experts) and n > 1 and cfg.num_experts % n == 0
        self.e_local = cfg.num_experts // n if self.ep else cfg.num_experts
        self.e0 = r * self.e_local if self.ep else 0
        self.moe_inter = cfg.intermediate_size if self.ep else self.local_inter
        if cfg.intermediate_size % n:
            raise ValueError("intermediate_size must be divisible by tensor_parallel_size")
        self.vocab_start, self.vocab_end = 0, cfg.vocab_size
        if n > 1 and cfg.vocab_size % n == 0:
            self.vocab_start, self.vocab_end = _shard(cfg.vocab_size, r, n)
        self.scale = 1.0 / math.sqrt(cfg.head_dim)
        self.max_pos = max_pos or cfg.max_position_embeddings
        self.cos_sin = cos_sin_table(cfg.rotary_dim, cfg.rope_theta, self.max_pos,
                                     cfg.rope_scaling, device=self.device)
        # ALiBi (position_embedding="alibi"): this rank's heads' slopes
        # (Megatron head split: rank r holds heads [r * local, (r + 1) * local))
        self.alibi = None
        if cfg.position_embedding == "alibi":
            from ..ops.reference import alibi_slopes
            h0 = r * self.local_heads
            self.alibi = alibi_slopes(cfg.num_heads)[h0:h0 + self.local_heads].float().contiguous().to(
                self.device)
        self.layers: List[SimpleNamespace] = []
        self.embed = None
        self.norm_w = None
        self.norm_b = None
        self.lm_head = None
        self.lm_head_b = None

    # ------------------------------------------------------------ weights
    def _alloc(self, *shape, dtype=None):
        return torch.empty(*shape, dtype=dtype or self.dtype, device=self.device)

    def allocate(self) -> None:
        c = self.cfg
        H, D = c.hidden_size, c.head_dim
        qkv_rows = (self.local_heads + 2 * self.local_kv_heads) * D
        # vocab-parallel embedding: each rank keeps the rows of its vocabulary
        # slice (the LM head's slice); lookups outside it give zero rows and
        # the cross-rank sum of the first reduction completes them
        self.embed = self._alloc(self.vocab_end - self.vocab_start, H)
        self.layers = []
        for _ in range(c.num_layers):
            L = SimpleNamespace()
            L.ln1 = self._alloc(H)
            L.ln1_b = self._alloc(H) if c.norm_type == "layernorm" else None
            L.wqkv = self._alloc(qkv_rows, H)
            L.bqkv = self._alloc(qkv_rows) if c.attention_bias else None
            L.wo = self._alloc(H, self.local_heads * D)
            L.bo = self._alloc(H) if c.norm_type == "layernorm" else None
            if not c.parallel_block:
                L.ln2 = self._alloc(H)
                L.ln2_b = None
            if c.num_experts:
                L.router = self._alloc(c.num_experts, H)
                L.w13 = self._alloc(self.e_local, 2 * self.moe_inter, H)
                L.w2 = self._alloc(self.e_local, H, self.moe_inter)
            elif c.hidden_act.startswith("gelu"):
                L.w1 = self._alloc(self.local_inter, H)
                L.b1 = self._alloc(self.local_inter) if c.mlp_bias else None
                L.w2 = self._alloc(H, self.local_inter)
                L.b2 = self._alloc(H) if c.mlp_bias else None
            else:
                L.w13 = self._alloc(2 * self.local_inter, H)
                L.w2 = self._alloc(H, self.local_inter)
            self.layers.append(L)
        self.norm_w = self._alloc(H)
        self.norm_b = self._alloc(H) if c.norm_type == "layernorm" else None
        self.lm_head = self._alloc(self.vocab_end - self.vocab_start, H)
        self.lm_head_b = self._alloc(self.vocab_end - self.vocab_start) if c.architecture == "phi" else None

    def named_parameters(self):
        yield "embed", self.embed
        for i, L in enumerate(self.layers):
            for k, v in vars(L).items():
                if isinstance(v, (ops.Fp8Weight, ops.Int8Weight)):
                    yield f"layers.{i}.{k}.q", v.q
                    yield f"layers.{i}.{k}.scale", v.scale
                elif isinstance(v, ops.Int4Weight):
                    yield f"layers.{i}.{k}.qp", v.qp
                    yield f"layers.{i}.{k}.sz", v.sz
                elif isinstance(v, ops.Nvfp4Weight):
                    yield f"layers.{i}.{k}.qp", v.qp
                    yield f"layers.{i}.{k}.sc", v.sc
                elif isinstance(v, torch.Tensor):
                    yield f"layers.{i}.{k}", v
        yield "norm", self.norm_w
        if self.norm_b is not None:
            yield "norm_b", self.norm_b
        yield "lm_head", self.lm_head
        if self.lm_head_b is not None:
            yield "lm_head_b", self.lm_head_b

    def init_dummy(self, seed: int = 0, std: float = 0.02) -> None:
        """Random N(0, std) init (norm weights 1, biases small); each rank's
        shard equals the matching slice of the single-rank tensor."""
        from ..parallel.dummy_init import fill_normal_sharded
        for name, t in self.named_parameters():
            leaf = name.split(".")[-1]
            if leaf in ("ln1", "ln2", "norm"):
                t.fill_(1.0)
                continue
            if leaf in ("ln1_b", "ln2_b", "norm_b"):
                t.zero_()
                continue
            fill_normal_sharded(t, self._full_spec(name, t), seed, tensor_id(name), std)

    def _full_spec(self, name: str, t: torch.Tensor):
        """(full_rows, full_cols, [(local_row_lo, full_row_lo, n)], col_lo) describing
        where this rank's shard sits inside the single-rank tensor, used so the
        dummy init is TP-invariant. Returns None for replicated tensors."""
        c = self.cfg
        r, n = self.tp.rank, self.tp.size
        D = c.head_dim
        leaf = name.split(".")[-1]
        if n == 1:
            return None
        if leaf in ("wqkv", "bqkv"):
            q0 = self.tp.rank * self.local_heads * D
            k0 = c.num_heads * D + self.kv_head_start * D
            v0 = (c.num_heads + c.num_kv_heads) * D + self.kv_head_start * D
            nq, nkv = self.local_heads * D, self.local_kv_heads * D
            full_rows = (c.num_heads + 2 * c.num_kv_heads) * D
            return ("rows", full_rows, [(0, q0, nq), (nq, k0, nkv), (nq + nkv, v0, nkv)])
        if leaf == "w13" and not c.num_experts:
            I = c.intermediate_size
            i0 = r * self.local_inter
            return ("rows", 2 * I, [(0, i0, self.local_inter),
                                    (self.local_inter, I + i0, self.local_inter)])
        if leaf in ("w13", "w2") and c.num_experts and self.ep:
            return ("exp", self.e0)
        if leaf == "w13" and c.num_experts:
            I = c.intermediate_size
            i0 = r * self.local_inter
            return ("rows3", 2 * I, [(0, i0, self.local_inter),
                                     (self.local_inter, I + i0, self.local_inter)])
        if leaf in ("w1", "b1"):
            return ("rows", c.intermediate_size, [(0, r * self.local_inter, self.local_inter)])
        if leaf == "wo":
            return ("cols", c.num_heads * D, r * self.local_heads * D)
        if leaf == "w2":
            if c.num_experts:
                return ("cols3", c.intermediate_size, r * self.local_inter)
            return ("cols", c.intermediate_size, r * self.local_inter)
        if leaf in ("lm_head", "lm_head_b", "embed") and self.vocab_end - self.vocab_start != c.vocab_size:
            return ("rows", c.vocab_size, [(0, self.vocab_start, self.vocab_end - self.vocab_start)])
        return None

    def quantize_int8(self) -> None:
        """W8A8: the dense projection weights (QKV, o_proj, gate_up / fc1,
        down / fc2) become per-output-feature int8; activations are
        quantized per token at every GEMM. Embedding, norms, LM head and MoE
        experts stay in the model dtype."""
        for L in self.layers:
            for name in ("wqkv", "wo", "w13", "w1", "w2"):
                w = getattr(L, name, None)
                if isinstance(w, torch.Tensor) and w.dim() == 2:
                    setattr(L, name, ops.int8_weight(w))
        if self.device.type == "cuda":
            torch.cuda.empty_cache()

    def quantize_int4(self, group: int = 128) -> None:
        """W4A16: the dense projection weights (QKV, o_proj, gate_up / fc1,
        down / fc2) become int4 codes with a bf16 scale and zero point per
        ``group`` input features (round to nearest; GPTQ / AWQ checkpoints
        arrive here dequantised and are re-packed with their own group size).
        Activations stay bf16. Embedding, norms, LM head and MoE experts stay
        in the model dtype. The kernel's groups are multiples of 64 input
        features: a per-channel checkpoint (group <= 0) uses one group per
        row, and a smaller group is widened to 64."""
        for L in self.layers:
            for name in ("wqkv", "wo", "w13", "w1", "w2"):
                w = getattr(L, name, None)
                if isinstance(w, torch.Tensor) and w.dim() == 2:
                    g = -(-w.shape[1] // 64) * 64 if group <= 0 else -(-group // 64) * 64
                    setattr(L, name, ops.int4.quantize(w, g))
        if self.device.type == "cuda":
            torch.cuda.empty_cache()

    def quantize_nvfp4(self) -> None:
        """NVFP4 weight storage for the dense projections (QKV, o_proj,
        gate_up / fc1, down / fc2): E2M1 codes with an E4M3 scale per 16
        input features and a per-tensor scale, expanded to bf16 in shared
        memory by the GEMM. Activations stay bf16."""
        for L in self.layers:
            for name in ("wqkv", "wo", "w13", "w1", "w2"):
                w = getattr(L, name, None)
                if isinstance(w, torch.Tensor) and w.dim() == 2:
                    setattr(L, name, ops.int4.quantize_nvfp4(w))
        if self.device.type == "cuda":
            torch.cuda.empty_cache()

    def quantize_fp8(self) -> None:
        """Replace the dense projection weights (QKV, o_proj, gate_up / fc1,
        down / fc2) by E4M3 weights with per-output-feature scales. The
        embedding, norms, LM head and MoE experts stay in the model dtype."""
        for L in self.layers:
            for name in ("wqkv", "wo", "w13", "w1", "w2"):
                w = getattr(L, name, None)
                if isinstance(w, torch.Tensor) and w.dim() == 2:
                    setattr(L, name, ops.fp8_weight(w))
        if self.device.type == "cuda":
            torch.cuda.empty_cache()

    def pad_k(self) -> None:
        """Zero-pad every dense projection weight whose input width is not a
        multiple of 8 (TMA rows must be 16-byte multiples; this happens for
        odd TP shard widths). Done once here, so a GEMM call pads only its
        activation."""
        for L in self.layers:
            for name in ("wqkv", "wo", "w13", "w1", "w2"):
                w = getattr(L, name, None)
                if isinstance(w, torch.Tensor) and w.dim() == 2 and w.shape[1] % 8:
                    setattr(L, name, torch.nn.functional.pad(w, (0, 8 - w.shape[1] % 8)).contiguous())

    def fuse_swiglu(self) -> None:
        """Store every dense gate/up weight interleaved (gate_i, up_i) so the
        SwiGLU activation runs in the GEMM epilogue (``ops.linear_swiglu``)."""
        for L in self.layers:
            w = getattr(L, "w13", None)
            if isinstance(w, torch.Tensor) and w.dim() == 2 and w.is_cuda:
                L.w13 = ops.interleave_gate_up(w)
                L.swiglu_fused = True
        if self.device.type == "cuda":
            torch.cuda.empty_cache()

    def _gate_up_act(self, L, x: torch.Tensor) -> torch.Tensor:
        if getattr(L, "swiglu_fused", False):
            return ops.linear_swiglu(x, L.w13)
        return ops.silu_and_mul(ops.linear(x, L.w13))

    def load_state(self, get: Callable[[str], Optional[torch.Tensor]]) -> None:
        """Fill weights from full (unsharded) HF-named tensors; ``get`` returns a
        CPU tensor or None. Slices the rank's shard before copying to device."""
        from .weights import load_hf_weights
        load_hf_weights(self, get)

    # ------------------------------------------------------------ forward
    def _norm(self, x, w, b, residual=None):
        if self.cfg.norm_type == "layernorm":
            return ops.layer_norm(x, w, b, self.cfg.rms_norm_eps, residual)
        return ops.rms_norm(x, w, self.cfg.rms_norm_eps, residual)

    def _attention(self, i: int, L, x: torch.Tensor, meta: AttnMeta, kv_cache: torch.Tensor,
                   reduce: bool = True):
        c = self.cfg
        qkv = ops.linear(x, L.wqkv)
        q = ops.qkv_rope_cache(qkv, meta.positions, self.cos_sin, kv_cache, i, meta.slot_mapping,
                               self.local_heads, self.local_kv_heads, c.head_dim, c.rotary_dim,
                               L.bqkv)
        a = ops.attention(q, kv_cache, i, meta, self.scale, c.sliding_window, self.alibi)
        a2 = a.reshape(a.shape[0], -1)
        if reduce:  # o_proj + cross-rank sum (one fused GEMM -> reduce-scatter under TP)
            return self.tp.linear_reduce(a2, L.wo)
        return ops.linear(a2, L.wo)

    def _reduce_slot(self, T: int):
        """Where a row-parallel GEMM should write its partial output: the
        fused TP backend hands out its NVLink-visible buffer (GEMM -> reduce
        with no copy); otherwise None (a fresh tensor)."""
        if self.tp.size > 1 and self.device.type == "cuda" and hasattr(self.tp, "reduce_buffer"):
            return self.tp.reduce_buffer(T, self.cfg.hidden_size)
        return None

    def _mlp(self, L, x: torch.Tensor, reduce: bool = True) -> torch.Tensor:
        c = self.cfg
        if c.num_experts:
            from ..parallel.moe import moe_forward
            y = moe_forward(self, L, x)
            return self.tp.reduce(y) if reduce else y
        if c.hidden_act.startswith("gelu"):
            h = ops.linear(x, L.w1, L.b1)
            h = ops.gelu_tanh(h)
            return self.tp.linear_reduce(h, L.w2) if reduce else ops.linear(h, L.w2)
        h = self._gate_up_act(L, x)
        if reduce:  # down_proj + cross-rank sum
            return self.tp.linear_reduce(h, L.w2)
        return ops.linear(h, L.w2)

    def _seq_parallel(self) -> bool:
        c = self.cfg
        return (getattr(self.tp, "sequence_parallel", False) and self.device.type == "cuda"
                and not c.parallel_block and c.norm_type != "layernorm")

    def _forward_seq_parallel(self, input_ids, meta: AttnMeta, kv_cache) -> torch.Tensor:
        """Tensor-parallel forward with a token-sharded residual: every
        row-parallel GEMM stores its partial locally, and one kernel per
        reduction sums this rank's token rows across ranks, adds the residual
        shard, applies the next norm and all-gathers the normalised rows
        (``tp.reduce_norm``). Returns the final-normed rows of logits_idx."""
        c = self.cfg
        T, H = int(input_ids.shape[0]), c.hidden_size
        if self.vocab_parallel:
            # partial lookups of every rank's vocabulary slice, summed by the
            # first reduction, which also norms and all-gathers them
            ops.embedding(input_ids, self.embed, self.vocab_start, out=self.tp.reduce_buffer(T, H))
            h = torch.zeros(T, H, dtype=self.embed.dtype, device=self.embed.device)
            x = self.tp.reduce_norm(T, h, self.layers[0].ln1, c.rms_norm_eps)
        else:
            h = ops.embedding(input_ids, self.embed)  # residual (own token rows kept current)
            x, _ = self._norm(h, self.layers[0].ln1, None)
        n = len(self.layers)
        for i, L in enumerate(self.layers):
            q = ops.qkv_rope_cache(ops.linear(x, L.wqkv), meta.positions, self.cos_sin, kv_cache, i,
                                   meta.slot_mapping, self.local_heads, self.local_kv_heads,
                                   c.head_dim, c.rotary_dim, L.bqkv)
            a = ops.attention(q, kv_cache, i, meta, self.scale, c.sliding_window, self.alibi)
            ops.linear(a.reshape(T, -1), L.wo, out=self.tp.reduce_buffer(T, H))
            x = self.tp.reduce_norm(T, h, L.ln2, c.rms_norm_eps)
            if c.num_experts:
                from ..parallel.moe import moe_forward
                moe_forward(self, L, x)  # the combine stores into the reduce buffer
            elif c.hidden_act.startswith("gelu"):
                g = ops.gelu_tanh(ops.linear(x, L.w1, L.b1))
                ops.linear(g, L.w2, L.b2 if self.tp.rank == 0 else None,
                           out=self.tp.reduce_buffer(T, H))
            else:
                ops.linear(self._gate_up_act(L, x), L.w2, out=self.tp.reduce_buffer(T, H))
            w_next = self.layers[i + 1].ln1 if i + 1 < n else self.norm_w
            x = self.tp.reduce_norm(T, h, w_next, c.rms_norm_eps)
        return x.index_select(0, meta.logits_idx)

    def forward(self, input_ids: torch.Tensor, meta: AttnMeta, kv_cache: torch.Tensor) -> torch.Tensor:
        """Returns final hidden states of the rows in ``meta.logits_idx``."""
        c = self.cfg
        if self._seq_parallel():
            return self._forward_seq_parallel(input_ids, meta, kv_cache)
        if self.vocab_parallel:  # VocabParallelEmbedding: zero rows off-slice, then the sum
            h = self.tp.reduce(ops.embedding(input_ids, self.embed, self.vocab_start))
        else:
            h = ops.embedding(input_ids, self.embed)
        residual = None
        for i, L in enumerate(self.layers):
            if c.parallel_block:
                x, _ = self._norm(h, L.ln1, L.ln1_b)
                a = self._attention(i, L, x, meta, kv_cache, reduce=False)
                m = self._mlp(L, x, reduce=False)
                s = a + m
                if self.tp.rank == 0:  # row-parallel biases are added once
                    if L.bo is not None:
                        s = s + L.bo
                    if getattr(L, "b2", None) is not None:
                        s = s + L.b2
                s = self.tp.reduce(s)
                h = h + s
                continue
            x, residual = self._norm(h, L.ln1, L.ln1_b, residual)
            a = self._attention(i, L, x, meta, kv_cache)
            x, residual = self._norm(a, L.ln2, L.ln2_b, residual)
            h = self._mlp(L, x)
        if c.parallel_block:
            last = h.index_select(0, meta.logits_idx)
            x, _ = self._norm(last, self.norm_w, self.norm_b)
            return x
        # only the sampled rows need the final norm and the LM head
        last_h = h.index_select(0, meta.logits_idx)
        last_r = residual.index_select(0, meta.logits_idx)
        x, _ = self._norm(last_h, self.norm_w, self.norm_b, last_r)
        return x

    @property
    def vocab_parallel(self) -> bool:
        return self.vocab_end - self.vocab_start != self.cfg.vocab_size

    def compute_logits(self, x: torch.Tensor, gather: bool = True) -> torch.Tensor:
        """fp32 logits; under tensor parallelism this rank's vocabulary slice
        [vocab_start, vocab_end), gathered over ranks when ``gather``."""
        logits = ops.linear(x, self.lm_head, self.lm_head_b).float()
        if gather and self.vocab_parallel:
            logits = self.tp.gather_vocab(logits)
        return logits
