"""numpy restatement of Weighted Correction Attention (TEST INFRASTRUCTURE ONLY).

Follows the reference ``src/cacheslide_vllm/wca.py`` (lines cited per function)
and ``src/cacheslide_vllm/policy.py:21-45``.  All reductions run in float64 as
the reference does; K/V are ``[token, head, dim]``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


def squared_deviation(cached, fresh) -> np.ndarray:
    """wca.py:55-62 -- per-token sum over heads and dims of (K' - K)^2."""
    d = fresh.astype(np.float64) - cached.astype(np.float64)
    return np.square(d).sum((1, 2))


def adaptation_weight(cached, fresh, epsilon=1e-8, clamp=False) -> np.ndarray:
    """wca.py:65-93 -- ||K' - K||^2 / (||K||^2 + eps), optional clamp."""
    num = squared_deviation(cached, fresh)
    den = np.square(cached.astype(np.float64)).sum((1, 2)) + epsilon
    with np.errstate(over="ignore", invalid="ignore", divide="ignore"):
        out = num / den
    return np.clip(out, 0, 1) if clamp else out


def mean_head_cosine(a, b, epsilon=1e-8) -> np.ndarray:
    """wca.py:96-112 -- amax-scaled unit vectors, clamped dot, head mean."""
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    sa = np.maximum(np.abs(a64).max(-1, keepdims=True), epsilon)
    sb = np.maximum(np.abs(b64).max(-1, keepdims=True), epsilon)
    a64, b64 = a64 / sa, b64 / sb
    tiny = np.finfo(np.float64).tiny
    na = np.maximum(np.sqrt(np.square(a64).sum(-1, keepdims=True)), tiny)
    nb = np.maximum(np.sqrt(np.square(b64).sum(-1, keepdims=True)), tiny)
    return np.clip(((a64 / na) * (b64 / nb)).sum(-1), -1, 1).mean(-1)


def select_top(deviation, available, slots: int) -> np.ndarray:
    """wca.py:202-215 -- the ``slots`` largest deviations among ``available``
    tokens, descending and stable (ties go to the lower token index)."""
    idx = np.nonzero(available)[0]
    order = np.argsort(-deviation[idx], kind="stable")
    return idx[order[: max(0, slots)]]


@dataclass
class OracleWCA:
    """wca.py:115-304 -- request-local WCA state machine."""

    correction_fraction: float = 0.26
    epsilon: float = 1e-8
    gate_interval: int = 4
    convergence_threshold: float = 0.12
    convergence_mode: str = "paper_cosine_lt"
    weight_update: str = "previous_layer"
    clamp_alpha: bool = False

    def initialize(self, cached, fresh, reused, mandatory):
        err = squared_deviation(cached, fresh)
        self.reused = reused.copy()
        self.mandatory = mandatory.copy()
        self.initial = err.copy()
        self.candidate = reused & (err > 0)
        self.budget = min(
            math.ceil(self.correction_fraction * int(reused.sum())),
            int(self.candidate.sum()),
        )
        self.selected = np.zeros_like(self.candidate)
        self.removed = np.zeros_like(self.candidate)
        self.alpha = adaptation_weight(cached, fresh, self.epsilon, self.clamp_alpha)
        self.last_layer = 1
        self._promote()
        return self

    @property
    def active(self):
        return np.nonzero(self.selected | self.mandatory)[0]

    def _promote(self):
        avail = self.candidate & ~self.selected & ~self.removed
        slots = max(0, self.budget - int(self.selected.sum()))
        chosen = select_top(self.initial, avail, slots)
        self.selected[chosen] = True
        return chosen

    def update(self, layer, cached_k, cached_v, fresh_k, fresh_v):
        idx = self.active
        old_k, old_v = cached_k[idx], cached_v[idx]
        nxt = adaptation_weight(old_k, fresh_k, self.epsilon, self.clamp_alpha)
        used = self.alpha[idx] if self.weight_update == "previous_layer" else nxt
        used = np.where(self.mandatory[idx], 1.0, used)
        w = used[:, None, None]
        fk = w * fresh_k.astype(np.float64) + (1 - w) * old_k.astype(np.float64)
        fv = w * fresh_v.astype(np.float64) + (1 - w) * old_v.astype(np.float64)
        removed = idx[:0]
        if layer % self.gate_interval == 0:
            cos = mean_head_cosine(fresh_k, old_k, self.epsilon)
            metric = cos if self.convergence_mode == "paper_cosine_lt" else 1 - cos
            removed = idx[self.selected[idx] & (metric < self.convergence_threshold)]
        self.alpha[idx] = nxt
        self.selected[removed] = False
        self.candidate[removed] = False
        self.removed[removed] = True
        promoted = self._promote()
        self.last_layer = layer
        return dict(
            indices=idx,
            fused_k=fk,
            fused_v=fv,
            alpha=used,
            removed=removed,
            promoted=promoted,
            next_indices=self.active,
        )
