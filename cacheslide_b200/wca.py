"""Weighted Correction Attention on B200 (reference ``wca.py``).

Same names, argument meaning and exception types as ``cacheslide_vllm.wca``:
float64 deviation/weight/cosine reductions, the ceil budget with a stable
top-budget selection, the previous-/same-layer weight orders, the cosine gate
every ``gate_interval`` layers and all-or-nothing commits.  The state lives
in device tensors; every computation is a CUDA kernel:

* ``initialize``: one fused reduction (deviation, alpha, candidates, counts)
  plus the block radix top-k;
* ``update``: one fused pass over the active rows (old-row gather, next
  weight, float64 blend, cast, optional cosine, optional paged scatter) and
  one commit kernel (weight store, gate removals, promotion).
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
from torch import Tensor

from . import _native as N
from .policy import WCAConfig, as_config, check_real

__all__ = [
    "WCAConfig",
    "WCANumericalError",
    "WCAState",
    "WCAUpdate",
    "adaptation_weight",
    "mean_head_cosine",
    "squared_deviation",
]


class WCANumericalError(ValueError):
    """Nonfinite WCA data or arithmetic that permits full-prefill recovery."""


def _kv(name: str, tensor: Tensor) -> None:
    """wca.py:26-32 (finiteness is checked by the kernels)."""
    if not isinstance(tensor, Tensor) or tensor.ndim != 3 or not tensor.is_floating_point():
        raise ValueError(f"{name} must be floating [token, head, dimension]")
    if min(tensor.shape[1:]) < 1:
        raise ValueError(f"{name} must have nonempty heads/dimension")


def _matching(name: str, tensor: Tensor, reference: Tensor) -> None:
    if (tensor.shape, tensor.dtype, tensor.device) != (
        reference.shape,
        reference.dtype,
        reference.device,
    ):
        raise ValueError(f"{name} shape, dtype and device must match its reference")
    _kv(name, tensor)


def _mask(name: str, tensor: Tensor, n: int, device: torch.device) -> None:
    if tensor.shape != (n,) or tensor.dtype != torch.bool or tensor.device != device:
        raise ValueError(f"{name} must be a bool [{n}] tensor on {device}")


def _inner(t: Tensor) -> Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


def _epsilon(epsilon) -> None:
    check_real("epsilon", epsilon)
    if epsilon <= 0:
        raise ValueError("epsilon must be finite and positive")


def _raise_numeric(bits: int, what: str) -> None:
    if bits & N.ST_INPUT_NONFINITE:
        raise WCANumericalError("cached_k/recomputed_k must have finite values")
    if bits & N.ST_NONFINITE:
        raise WCANumericalError(what)


def _raise_update(bits: int) -> None:
    if bits & N.ST_SLOT_RANGE:
        raise ValueError("paged KV slot outside the arena")
    if bits & (N.ST_NONFINITE | N.ST_INPUT_NONFINITE):
        raise WCANumericalError("weighted K/V overflowed the cache dtype")


def _deviation(cached: Tensor, fresh: Tensor, epsilon: float, clamp: bool, want_alpha: bool):
    device = N.require_cuda(cached, fresh)
    c, f = _inner(cached), _inner(fresh)
    n = c.shape[0]
    dev = torch.empty(n, dtype=torch.float64, device=device)
    alpha = torch.empty_like(dev) if want_alpha else None
    status = N.Status(device)
    N.check(
        N.load().cs_wca_deviation(
            c.data_ptr(), c.stride(0), c.stride(1), None, f.data_ptr(), f.stride(0), f.stride(1),
            n, c.shape[1], c.shape[2], N.DTYPES[c.dtype], float(epsilon), int(clamp),
            dev.data_ptr(), N.ptr(alpha), status.ptr, N.stream_of(device),
        ),
        "cs_wca_deviation",
    )
    return dev, alpha, status.read()


def squared_deviation(cached_k: Tensor, recomputed_k: Tensor) -> Tensor:
    """Per-token squared K error, summed over all heads and dims (wca.py:55-62)."""
    _kv("cached_k", cached_k)
    _matching("recomputed_k", recomputed_k, cached_k)
    dev, _, bits = _deviation(cached_k, recomputed_k, 1.0, False, False)
    _raise_numeric(bits, "squared deviation overflowed float64")
    return dev


def adaptation_weight(
    cached_k: Tensor,
    recomputed_k: Tensor,
    *,
    epsilon: float = 1e-8,
    clamp: bool = False,
) -> Tensor:
    """Raw ||K_new-K_cache||^2 / (||K_cache||^2 + epsilon) per token (wca.py:65-93)."""
    _kv("cached_k", cached_k)
    _matching("recomputed_k", recomputed_k, cached_k)
    _epsilon(epsilon)
    if type(clamp) is not bool:
        raise ValueError("clamp must be a boolean")
    _, alpha, bits = _deviation(cached_k, recomputed_k, epsilon, clamp, True)
    _raise_numeric(bits, "adaptation weight overflowed; inspect the K magnitudes")
    return alpha


def mean_head_cosine(a: Tensor, b: Tensor, *, epsilon: float = 1e-8) -> Tensor:
    """Mean cosine over heads; zero-norm heads contribute zero (wca.py:96-112)."""
    _kv("a", a)
    _matching("b", b, a)
    _epsilon(epsilon)
    device = N.require_cuda(a, b)
    a_, b_ = _inner(a), _inner(b)
    out = torch.empty(a_.shape[0], dtype=torch.float64, device=device)
    status = N.Status(device)
    N.check(
        N.load().cs_wca_cosine(
            a_.data_ptr(), a_.stride(0), a_.stride(1), b_.data_ptr(), b_.stride(0), b_.stride(1),
            None, a_.shape[0], a_.shape[1], a_.shape[2], N.DTYPES[a_.dtype], float(epsilon),
            out.data_ptr(), status.ptr, N.stream_of(device),
        ),
        "cs_wca_cosine",
    )
    _raise_numeric(status.read(), "cosine inputs must be finite")
    return out


@dataclass(frozen=True)
class WCAUpdate:
    """Corrected current-layer rows and selection changes (wca.py:115-125)."""

    indices: Tensor
    fused_k: Tensor
    fused_v: Tensor
    alpha: Tensor
    removed_indices: Tensor
    promoted_indices: Tensor
    next_indices: Tensor


@dataclass
class WCAState:
    """Request-local WCA state on the device (wca.py:128-304)."""

    config: WCAConfig
    reused_mask: Tensor
    mandatory_mask: Tensor
    initial_deviation: Tensor
    candidate_mask: Tensor
    selected_mask: Tensor
    removed_mask: Tensor
    alpha: Tensor
    budget: int
    last_layer: int = 1

    @classmethod
    def initialize(
        cls,
        cached_k: Tensor,
        recomputed_k: Tensor,
        reused_mask: Tensor,
        mandatory_mask: Tensor,
        config: WCAConfig | None = None,
    ) -> WCAState:
        config = as_config(config)
        _kv("cached_k", cached_k)
        _matching("recomputed_k", recomputed_k, cached_k)
        n = cached_k.shape[0]
        device = N.require_cuda(cached_k)
        _mask("reused_mask", reused_mask, n, cached_k.device)
        _mask("mandatory_mask", mandatory_mask, n, cached_k.device)
        if bool(((~reused_mask) & (~mandatory_mask)).any()):
            raise ValueError("every dynamic/non-reused token must be mandatory")
        c, f = _inner(cached_k), _inner(recomputed_k)
        reused = reused_mask.clone()
        dev = torch.empty(n, dtype=torch.float64, device=device)
        alpha = torch.empty_like(dev)
        candidate = torch.empty(n, dtype=torch.bool, device=device)
        selected = torch.empty_like(candidate)
        removed = torch.empty_like(candidate)
        counts = torch.empty(2, dtype=torch.int64, device=device)
        status = N.Status(device)
        N.check(
            N.load().cs_wca_initialize(
                c.data_ptr(), c.stride(0), c.stride(1), f.data_ptr(), f.stride(0), f.stride(1),
                n, c.shape[1], c.shape[2], N.DTYPES[c.dtype], reused.data_ptr(),
                float(config.epsilon), int(config.clamp_alpha), dev.data_ptr(), alpha.data_ptr(),
                candidate.data_ptr(), selected.data_ptr(), removed.data_ptr(),
                counts.data_ptr(), status.ptr, N.stream_of(device),
            ),
            "cs_wca_initialize",
        )
        _raise_numeric(status.read(), "squared deviation overflowed float64")
        reused_count, candidate_count = counts.tolist()
        budget = min(math.ceil(config.correction_fraction * reused_count), candidate_count)
        state = cls(
            config=config,
            reused_mask=reused,
            mandatory_mask=mandatory_mask.clone(),
            initial_deviation=dev,
            candidate_mask=candidate,
            selected_mask=selected,
            removed_mask=removed,
            alpha=alpha,
            budget=budget,
        )
        state._promote()
        return state

    @property
    def active_indices(self) -> Tensor:
        """Sorted global token indices to compute at the next layer."""
        return (self.selected_mask | self.mandatory_mask).nonzero().flatten()

    def active_rows_device(self, capacity: int, status: Tensor | None = None):
        """The next layer's active rows without a host read.

        Returns device tensors ``rows`` (int64 ``[capacity]``: ``active_indices``
        then -1), ``association`` (uint8 ``[capacity]``: the row is selected and
        not mandatory, runtime.py:448-454) and ``count`` (int64 ``[1]``), all
        written by one kernel on the current stream.  Pass ``count`` as
        ``AttnParams.nq_dev`` to run the next prefill on these rows.  Rows past
        ``capacity`` are dropped and set CS_ST_SLOT_RANGE in ``status``.
        """
        dev = self.selected_mask.device
        n = self.selected_mask.numel()
        rows = torch.empty(max(capacity, 1), dtype=torch.int64, device=dev)[:capacity]
        assoc = torch.empty(max(capacity, 1), dtype=torch.uint8, device=dev)[:capacity]
        count = torch.empty(1, dtype=torch.int64, device=dev)
        st = status.data_ptr() if status is not None else None
        N.check(N.load().cs_wca_active_rows(
            self.selected_mask.data_ptr(), self.mandatory_mask.data_ptr(), n, capacity,
            rows.data_ptr(), assoc.data_ptr(), count.data_ptr(), st, N.stream_of(dev)),
            "cs_wca_active_rows")
        return rows, assoc, count

    @property
    def selected_indices(self) -> Tensor:
        return self.selected_mask.nonzero().flatten()

    def _commit(self, indices, next_alpha, cosine) -> tuple[Tensor, Tensor]:
        device = self.selected_mask.device
        n = self.selected_mask.numel()
        a = 0 if indices is None else indices.numel()
        removed = torch.empty(max(a, 1), dtype=torch.int64, device=device)
        promoted = torch.empty(max(min(self.budget, n), 1), dtype=torch.int64, device=device)
        counts = torch.zeros(2, dtype=torch.int64, device=device)
        status = N.Status(device)
        distance = self.config.convergence_mode != "paper_cosine_lt"
        N.check(
            N.load().cs_wca_commit(
                N.ptr(indices), a, N.ptr(next_alpha), N.ptr(cosine),
                float(self.config.convergence_threshold), int(distance), n, self.budget,
                self.initial_deviation.data_ptr(), self.alpha.data_ptr(),
                self.candidate_mask.data_ptr(), self.selected_mask.data_ptr(),
                self.removed_mask.data_ptr(), removed.data_ptr(), promoted.data_ptr(),
                counts.data_ptr(), status.ptr, N.stream_of(device),
            ),
            "cs_wca_commit",
        )
        n_removed, n_promoted = counts.tolist()
        return removed[:n_removed], promoted[:n_promoted]

    def _promote(self) -> Tensor:
        return self._commit(None, None, None)[1]

    def _check_update(self, layer_index, cached_k, cached_v, recomputed_k, recomputed_v,
                      computed_indices):
        """Argument checks of ``update`` (wca.py:217-250); returns the active
        indices and the row views the kernels read."""
        if layer_index != self.last_layer + 1:
            raise ValueError("layers must update consecutively after full layer one")
        _kv("cached_k", cached_k)
        _matching("cached_v", cached_v, cached_k)
        if cached_k.shape[0] != self.reused_mask.numel():
            raise ValueError("cache token count differs from the request")
        if cached_k.device != self.reused_mask.device:
            raise ValueError("cache device differs from the request")
        indices = self.active_indices
        if computed_indices is not None:
            if (
                computed_indices.dtype != torch.long
                or computed_indices.device != indices.device
                or not torch.equal(computed_indices, indices)
            ):
                raise ValueError("computed_indices must equal sorted active_indices")
        a = indices.numel()
        expected = (a, *cached_k.shape[1:])
        for name, t in (("recomputed_k", recomputed_k), ("recomputed_v", recomputed_v)):
            if (tuple(t.shape), t.dtype, t.device) != (expected, cached_k.dtype, cached_k.device):
                raise ValueError(f"{name} shape, dtype and device must match its reference")
            _kv(name, t)
        N.require_cuda(cached_k)
        ck, cv = _inner(cached_k), _inner(cached_v)
        if ck.stride() != cv.stride():
            cv = cv.contiguous()
            ck = ck.contiguous()
        fk, fv = _inner(recomputed_k), _inner(recomputed_v)
        if fk.stride() != fv.stride():
            fk, fv = fk.contiguous(), fv.contiguous()
        return indices, ck, cv, fk, fv

    def _blend(self, indices, ck, cv, fk, fv, *, same_layer: bool, cosine, paged,
               alpha: Tensor | None = None, check: bool = True):
        """One fused pass over the active rows (cs_wca_update): next weight,
        float64 blend with the used weight (``alpha[index]`` unless
        ``same_layer``; mandatory rows 1), cast, optional cosine and paged
        scatter.  Returns (fused_k, fused_v, next_alpha, used_alpha), plus the
        status bits instead of raising when ``check`` is false."""
        alpha = self.alpha if alpha is None else alpha
        device = ck.device
        a = indices.numel()
        fused_k = torch.empty((a, *ck.shape[1:]), dtype=ck.dtype, device=device)
        fused_v = torch.empty_like(fused_k)
        next_alpha = torch.empty(a, dtype=torch.float64, device=device)
        used = torch.empty_like(next_alpha)
        kv = slots = None
        if paged is not None:
            arena, slots = paged
            kv = arena.device_view()
        status = N.Status(device)
        N.check(
            N.load().cs_wca_update(
                ck.data_ptr(), cv.data_ptr(), ck.stride(0), ck.stride(1), fk.data_ptr(),
                fv.data_ptr(), fk.stride(0), fk.stride(1), indices.data_ptr(), a,
                ck.shape[1], ck.shape[2], N.DTYPES[ck.dtype], alpha.data_ptr(),
                self.mandatory_mask.data_ptr(), int(same_layer),
                float(self.config.epsilon), int(self.config.clamp_alpha), fused_k.data_ptr(),
                fused_v.data_ptr(), next_alpha.data_ptr(), used.data_ptr(), N.ptr(cosine),
                None if kv is None else ctypes.byref(kv), N.ptr(slots),
                status.ptr, N.stream_of(device),
            ),
            "cs_wca_update",
        )
        bits = status.read()
        if not check:
            return fused_k, fused_v, next_alpha, used, bits
        _raise_update(bits)
        return fused_k, fused_v, next_alpha, used

    def update(
        self,
        layer_index: int,
        cached_k: Tensor,
        cached_v: Tensor,
        recomputed_k: Tensor,
        recomputed_v: Tensor,
        computed_indices: Tensor | None = None,
        *,
        paged=None,
    ) -> WCAUpdate:
        """Fuse sparse recomputed rows against full current-layer cached K/V.

        ``paged=(NativePagedKV, slots)`` additionally writes the fused rows to
        their paged slots in the same kernel (blend + scatter).
        """
        indices, ck, cv, fk, fv = self._check_update(
            layer_index, cached_k, cached_v, recomputed_k, recomputed_v, computed_indices)
        gate = layer_index % self.config.gate_interval == 0
        cosine = torch.empty(indices.numel(), dtype=torch.float64,
                             device=ck.device) if gate else None
        fused_k, fused_v, next_alpha, used = self._blend(
            indices, ck, cv, fk, fv, same_layer=self.config.weight_update == "same_layer",
            cosine=cosine, paged=paged)
        removed, promoted = self._commit(indices, next_alpha, cosine)
        self.last_layer = layer_index
        return WCAUpdate(
            indices=indices,
            fused_k=fused_k,
            fused_v=fused_v,
            alpha=used,
            removed_indices=removed,
            promoted_indices=promoted,
            next_indices=self.active_indices,
        )
