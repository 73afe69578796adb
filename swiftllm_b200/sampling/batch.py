"""Batch sampler used by the engine each step.

Per sample row: penalties (if the batch has any) -> temperature -> min-p ->
top-k -> top-p -> Philox draw, on the GPU in one fused kernel
(``_C.sample``); on CPU tensors the same maths runs row by row through the
C++ oracle (``_core.sample_row``). The uniform draw of row r is
Philox4x32-10(key, counter) with
  key = (seed, 0x5EED), counter = (step_idx, 0)     for seeded requests,
  key = (engine seed, 0xA11), counter = (step, r)   otherwise,
so seeded requests are reproducible regardless of batch composition.
"""

from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import numpy as np
import torch

from .. import _core
from ..parallel.dummy_init import mix_key


def row_keys(seed: np.ndarray, step_idx: np.ndarray, engine_seed: int,
             step: int) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(key uint64, c0 uint32, c1 uint32) per row."""
    n = seed.shape[0]
    seed = np.asarray(seed, dtype=np.int64)
    seeded = seed >= 0
    # mix_key(seed, 0x5EED) for seeded rows, vectorised: (seed << 32) | tid
    sk = ((seed.astype(np.uint64) & np.uint64(0xFFFFFFFF)) << np.uint64(32)) | np.uint64(0x5EED)
    keys = np.where(seeded, sk, np.uint64(mix_key(engine_seed, 0xA11))).astype(np.uint64)
    c0 = np.where(seeded, np.asarray(step_idx, dtype=np.int64) & 0xFFFFFFFF,
                  step & 0xFFFFFFFF).astype(np.uint32)
    c1 = np.where(seeded, 0, np.arange(n)).astype(np.uint32)
    return keys, c0, c1


class BatchSampler:
    def __init__(self, vocab_size: int, engine_seed: int, device: torch.device):
        self.vocab = vocab_size
        self.seed = engine_seed
        self.device = torch.device(device)
        self.step = 0

    @staticmethod
    def penalty_csr(n: int, rep: np.ndarray, pres: np.ndarray, freq: np.ndarray,
                    hist: Callable[[int], Tuple[np.ndarray, np.ndarray]]):
        """Per sample row, the distinct tokens a penalty touches with their
        output counts: (offsets [n + 1], tokens, out_counts) int32. Rows
        without penalties are empty; presence/frequency only see generated
        tokens (count > 0), repetition also the prompt's."""
        offs = np.zeros(n + 1, dtype=np.int32)
        toks, cnts = [], []
        for r in range(n):
            if rep[r] == 1.0 and pres[r] == 0.0 and freq[r] == 0.0:
                offs[r + 1] = offs[r]
                continue
            prompt, output = hist(r)
            uo, co = np.unique(np.asarray(output, dtype=np.int64), return_counts=True)
            if rep[r] != 1.0 and len(prompt):
                up = np.setdiff1d(np.unique(np.asarray(prompt, dtype=np.int64)), uo,
                                  assume_unique=True)
                t = np.concatenate([uo, up])
                c = np.concatenate([co, np.zeros(up.size, dtype=co.dtype)])
            else:
                t, c = uo, co
            toks.append(t.astype(np.int32))
            cnts.append(c.astype(np.int32))
            offs[r + 1] = offs[r] + t.size
        tk = np.concatenate(toks) if toks else np.zeros(0, np.int32)
        ct = np.concatenate(cnts) if cnts else np.zeros(0, np.int32)
        return offs, tk, ct

    def _penalize(self, logits: torch.Tensor, b, rows: np.ndarray,
                  history: Callable[[int], Tuple[np.ndarray, np.ndarray]]) -> torch.Tensor:
        """Repetition/frequency/presence penalties on a private copy of each
        sample row's logits; history(seq_id) -> (prompt_ids, output_ids).
        On the GPU: one gather, one host->device copy of the penalty table
        (CSR) and one kernel for the whole batch."""
        rep = np.asarray(b.repetition_penalty, dtype=np.float32)
        pres = np.asarray(b.presence_penalty, dtype=np.float32)
        freq = np.asarray(b.frequency_penalty, dtype=np.float32)
        lidx = np.asarray(b.sample_logit_idx)
        tgt = np.asarray(b.sample_target_seq)
        seq_ids = np.asarray(b.seq_ids)
        srow = np.asarray(b.sample_seq_row)
        n = lidx.shape[0]
        sid = lambda r: int(tgt[r]) if tgt[r] >= 0 else int(seq_ids[srow[r]])  # noqa: E731
        out = logits.index_select(0, torch.from_numpy(lidx.astype(np.int64)).to(logits.device))
        offs, tk, ct = self.penalty_csr(n, rep, pres, freq, lambda r: history(sid(r)))
        if not out.is_cuda:
            V = out.shape[1]
            for r in range(n):
                a, e = int(offs[r]), int(offs[r + 1])
                if a == e:
                    continue
                t = torch.from_numpy(tk[a:e].astype(np.int64))
                c = torch.from_numpy(ct[a:e].astype(np.float32))
                ok = (t >= 0) & (t < V)
                t, c = t[ok], c[ok]
                v = out[r, t]
                if rep[r] != 1.0:
                    v = torch.where(v > 0, v / float(rep[r]), v * float(rep[r]))
                v = v - torch.where(c > 0, float(freq[r]) * c + float(pres[r]), torch.zeros_like(c))
                out[r, t] = v
            return out
        from ..ops import cuda_ext
        dev = out.device
        ints = torch.from_numpy(np.concatenate([offs, tk, ct]).astype(np.int32)).to(dev, non_blocking=True)
        fp = torch.from_numpy(np.concatenate([rep, pres, freq]).astype(np.float32)).to(dev, non_blocking=True)
        o_t = ints[:n + 1]
        t_t = ints[n + 1:n + 1 + tk.size]
        c_t = ints[n + 1 + tk.size:]
        cuda_ext().apply_penalties(out, o_t, t_t, c_t, fp)
        from .. import ops as _ops
        _ops._count()
        return out

    def __call__(self, logits: torch.Tensor, b,
                 history: Optional[Callable[[int], Tuple[np.ndarray, np.ndarray]]] = None
                 ) -> Tuple[np.ndarray, np.ndarray]:
        """Returns (tokens int32 [rows], logprobs float32 [rows])."""
        self.step += 1
        n = int(b.num_sample_rows)
        if n == 0:
            return np.zeros(0, np.int32), np.zeros(0, np.float32)
        lidx = np.asarray(b.sample_logit_idx, dtype=np.int32)
        if hasattr(logits, "tokens"):  # vocab-parallel greedy result (all rows greedy)
            both = torch.stack([logits.tokens.view(torch.float32), logits.lps]).cpu().numpy()
            return both[0].view(np.int32)[lidx].copy(), both[1][lidx].copy()
        if b.any_penalty and history is not None:
            rows_logits = self._penalize(logits, b, lidx, history)
            lidx = np.arange(n, dtype=np.int32)
        else:
            rows_logits = logits
        temp = np.asarray(b.temperature, dtype=np.float32)
        top_p = np.asarray(b.top_p, dtype=np.float32)
        top_k = np.asarray(b.top_k, dtype=np.int32)
        min_p = np.asarray(b.min_p, dtype=np.float32)
        keys, c0, c1 = row_keys(np.asarray(b.seed), np.asarray(b.step_idx), self.seed, self.step)
        if rows_logits.is_cuda:
            from ..ops import cuda_ext
            C = cuda_ext()
            f = torch.from_numpy(np.stack([temp, top_p, min_p]).astype(np.float32))
            i = torch.from_numpy(np.stack([lidx, top_k, c0.view(np.int32), c1.view(np.int32)]))
            k = torch.from_numpy(keys.view(np.int64))
            dev = rows_logits.device
            tokens = torch.empty(n, dtype=torch.int32, device=dev)
            lps = torch.empty(n, dtype=torch.float32, device=dev)
            C.sample(tokens, lps, rows_logits, f.to(dev, non_blocking=True),
                     i.to(dev, non_blocking=True), k.to(dev, non_blocking=True),
                     bool(b.any_random))
            from .. import ops as _ops
            _ops._count()
            both = torch.stack([tokens.view(torch.float32), lps]).cpu().numpy()
            return both[0].view(np.int32).copy(), both[1].copy()
        lg = rows_logits.float().numpy()
        toks = np.empty(n, dtype=np.int32)
        lps = np.empty(n, dtype=np.float32)
        for r in range(n):
            u = _core.philox_uniform(int(keys[r]), int(c0[r]), int(c1[r]))
            p = _core.SampleParams(temperature=float(temp[r]), top_p=float(top_p[r]),
                                   top_k=int(top_k[r]), min_p=float(min_p[r]))
            t, lp = _core.sample_row(lg[lidx[r]], p, u)
            toks[r], lps[r] = t, lp
        return toks, lps
