"""Public sampling helpers (host side) and the engine's batch sampler.

Parity: python/swiftllm/sampling.py (Sampler classes :13-231,
SamplingStrategy :233-362, create_sampler :372-397) and the Rust
SamplerChain (crates/swiftllm-core/src/sampling/strategies.rs:360-439).

Differences by design:
  * one stage order everywhere (penalties -> temperature -> min-p -> top-k
    -> top-p -> draw), the same one the GPU kernel uses; the reference's
    Python helper applies min-p last and its Rust chain applies it first;
  * a per-strategy counter-based generator (Philox4x32-10, keyed by the
    seed) instead of re-seeding numpy's global generator (sampling.py:256-259
    makes every strategy share and reset one global state);
  * penalties count prompt tokens for the repetition penalty only.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import numpy as np

from .. import _core


def _as_logits(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32).reshape(-1))


class Sampler:
    """Base class: ``sampler(logits, token_ids) -> (token_id, logprob)``."""

    def __init__(self, seed: Optional[int] = None):
        self._key = (0x5EED if seed is None else int(seed)) & 0xFFFFFFFFFFFFFFFF
        self._step = 0

    def _uniform(self) -> float:
        u = _core.philox_uniform(self._key, self._step & 0xFFFFFFFF, self._step >> 32)
        self._step += 1
        return u

    def _sample(self, logits, params: "_core.SampleParams",
                token_ids: Optional[Sequence[int]] = None) -> Tuple[int, float]:
        out = np.asarray(token_ids if token_ids else [], dtype=np.int32)
        tok, lp = _core.sample_row(_as_logits(logits), params, self._uniform(),
                                   np.zeros(0, np.int32), out)
        return int(tok), float(lp)

    def __call__(self, logits, token_ids: Optional[List[int]] = None) -> Tuple[int, float]:
        raise NotImplementedError


class GreedySampler(Sampler):
    def __call__(self, logits, token_ids=None):
        return self._sample(logits, _core.SampleParams(temperature=0.0), None)


class TemperatureSampler(Sampler):
    def __init__(self, temperature: float = 1.0, seed: Optional[int] = None):
        super().__init__(seed)
        if temperature <= 0:
            raise ValueError(f"Temperature must be positive, got {temperature}")
        self.temperature = temperature

    def __call__(self, logits, token_ids=None):
        return self._sample(logits, _core.SampleParams(temperature=self.temperature), None)


class TopKSampler(Sampler):
    def __init__(self, k: int, temperature: float = 1.0, seed: Optional[int] = None):
        super().__init__(seed)
        if k <= 0:
            raise ValueError(f"k must be positive, got {k}")
        self.k, self.temperature = k, temperature

    def __call__(self, logits, token_ids=None):
        return self._sample(logits, _core.SampleParams(temperature=self.temperature, top_k=self.k))


class TopPSampler(Sampler):
    def __init__(self, p: float, temperature: float = 1.0, seed: Optional[int] = None):
        super().__init__(seed)
        if not 0 < p <= 1:
            raise ValueError(f"p must be in (0, 1], got {p}")
        self.p, self.temperature = p, temperature

    def __call__(self, logits, token_ids=None):
        return self._sample(logits, _core.SampleParams(temperature=self.temperature, top_p=self.p))


class MinPSampler(Sampler):
    def __init__(self, min_p: float, temperature: float = 1.0, seed: Optional[int] = None):
        super().__init__(seed)
        if not 0 <= min_p <= 1:
            raise ValueError(f"min_p must be in [0, 1], got {min_p}")
        self.min_p, self.temperature = min_p, temperature

    def __call__(self, logits, token_ids=None):
        return self._sample(logits, _core.SampleParams(temperature=self.temperature,
                                                       min_p=self.min_p))


class BeamSearchSampler(Sampler):
    """Single-step view of beam search: the best token and its logprob. The
    engine keeps full beams (``SamplingParams.use_beam_search``)."""

    def __init__(self, beam_width: int, length_penalty: float = 1.0):
        super().__init__(None)
        self.beam_width = beam_width
        self.length_penalty = length_penalty

    def __call__(self, logits, token_ids=None):
        return self._sample(logits, _core.SampleParams(temperature=0.0))

    def topk(self, logits) -> List[Tuple[int, float]]:
        x = _as_logits(logits).astype(np.float64)
        lp = x - (np.log(np.exp(x - x.max()).sum()) + x.max())
        idx = np.argsort(-lp, kind="stable")[: self.beam_width]
        return [(int(i), float(lp[i])) for i in idx]


@dataclass
class SamplingStrategy:
    temperature: float = 1.0
    top_k: int = -1
    top_p: float = 1.0
    min_p: float = 0.0
    presence_penalty: float = 0.0
    frequency_penalty: float = 0.0
    repetition_penalty: float = 1.0
    seed: Optional[int] = None
    _sampler: Sampler = field(default=None, init=False, repr=False)

    def __post_init__(self):
        self._sampler = Sampler(self.seed)

    @property
    def params(self) -> "_core.SampleParams":
        return _core.SampleParams(temperature=self.temperature, top_p=self.top_p,
                                  top_k=self.top_k, min_p=self.min_p,
                                  presence_penalty=self.presence_penalty,
                                  frequency_penalty=self.frequency_penalty,
                                  repetition_penalty=self.repetition_penalty)

    def apply_penalties(self, logits, token_ids: List[int],
                        prompt_ids: Optional[List[int]] = None) -> np.ndarray:
        """Returns penalised logits. Repetition: divide positive / multiply
        negative logits of seen tokens; frequency: subtract penalty x count;
        presence: subtract penalty once per generated token id."""
        x = _as_logits(logits).copy()
        seen = set(token_ids or []) | set(prompt_ids or [])
        if self.repetition_penalty != 1.0:
            for t in seen:
                if 0 <= t < x.size:
                    x[t] = x[t] / self.repetition_penalty if x[t] > 0 else x[t] * self.repetition_penalty
        counts = {}
        for t in token_ids or []:
            counts[t] = counts.get(t, 0) + 1
        for t, c in counts.items():
            if 0 <= t < x.size:
                x[t] -= self.frequency_penalty * c + self.presence_penalty
        return x

    def sample(self, logits, token_ids: Optional[List[int]] = None) -> Tuple[int, float]:
        return self._sampler._sample(logits, self.params, token_ids)


def create_sampler(temperature: float = 1.0, top_k: int = -1, top_p: float = 1.0,
                   min_p: float = 0.0, **kwargs) -> SamplingStrategy:
    return SamplingStrategy(temperature=temperature, top_k=top_k, top_p=top_p, min_p=min_p,
                            **kwargs)


__all__ = ["Sampler", "GreedySampler", "TemperatureSampler", "TopKSampler", "TopPSampler",
           "MinPSampler", "BeamSearchSampler", "SamplingStrategy", "create_sampler"]
