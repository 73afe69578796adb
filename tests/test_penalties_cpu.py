"""Batched penalties (one table, one pass over the batch) against the C++
sampling oracle, which applies repetition / frequency / presence penalties
row by row from the raw histories."""

import numpy as np
import torch

from swiftllm_b200 import _core
from swiftllm_b200.sampling.batch import BatchSampler


def _case(seed=0, n=6, V=50):
    rng = np.random.default_rng(seed)
    logits = rng.normal(size=(n, V)).astype(np.float32)
    hist = [(rng.integers(0, V, size=rng.integers(0, 12)).astype(np.int32),
             rng.integers(0, V, size=rng.integers(0, 20)).astype(np.int32)) for _ in range(n)]
    rep = np.array([1.0, 1.3, 1.0, 2.0, 1.0, 0.8], dtype=np.float32)[:n]
    pres = np.array([0.0, 0.0, 0.5, 0.2, 0.0, 1.0], dtype=np.float32)[:n]
    freq = np.array([0.0, 0.0, 0.3, 0.0, 0.7, 0.4], dtype=np.float32)[:n]
    return logits, hist, rep, pres, freq


def apply_csr(logits, offs, tk, ct, rep, pres, freq):
    out = torch.from_numpy(logits.copy())
    for r in range(out.shape[0]):
        a, e = int(offs[r]), int(offs[r + 1])
        for t, c in zip(tk[a:e], ct[a:e]):
            v = float(out[r, int(t)])
            if rep[r] != 1.0:
                v = v / rep[r] if v > 0 else v * rep[r]
            if c > 0:
                v -= freq[r] * c + pres[r]
            out[r, int(t)] = float(v)
    return out


def test_penalty_table_matches_oracle():
    logits, hist, rep, pres, freq = _case()
    n, V = logits.shape
    offs, tk, ct = BatchSampler.penalty_csr(n, rep, pres, freq, lambda r: hist[r])
    got = apply_csr(logits, offs, tk, ct, rep, pres, freq)
    for r in range(n):
        p = _core.SampleParams(temperature=0.0, repetition_penalty=float(rep[r]),
                               presence_penalty=float(pres[r]), frequency_penalty=float(freq[r]))
        tok, lp = _core.sample_row(logits[r], p, 0.0, hist[r][0], hist[r][1])
        want_lp = torch.log_softmax(got[r].double(), -1)
        assert int(torch.argmax(got[r])) == tok
        assert abs(float(want_lp[tok]) - lp) < 1e-4
