"""KV-head tensor-parallel WCA (the Llama-70B TP8 layout of CacheSlide).

Under KV-head tensor parallelism each rank holds the K/V of ``heads`` of the
model's ``heads_total`` KV heads (and their query heads).  Attention needs no
exchange: a rank attends its own heads.  WCA does: the squared deviation,
the norm of the adaptation weight and the head-mean cosine are sums over all
heads (reference ``wca.py:55-112``), so a rank that reduced only its own
heads would select different tokens than its peers.  ``ShardedWCAState``
keeps every rank on the same selection:

* each rank computes its shard's per-row partial sums on the device
  (``cs_wca_row_sums``: deviation, norm and cosine / heads_total);
* one all-reduce per step sums them over the ranks (``[2, n]`` float64 at
  initialize, ``[2, a]`` or ``[3, a]`` per layer);
* from the complete sums every rank derives the same weights, candidates,
  budget, selection, gate removals and promotions (the same kernels on the
  same inputs: ``cs_wca_weights``, ``cs_wca_commit``), and blends and scatters
  only its own heads (``cs_wca_update`` with the complete weights).

The state, the commit and the blend are those of ``WCAState``; only the head
reductions change.  The group is any ``torch.distributed`` process group
(NCCL for device tensors).
"""

from __future__ import annotations

import math

import torch
import torch.distributed as dist
from torch import Tensor

from . import _native as N
from .policy import WCAConfig, as_config
from .wca import (WCAState, WCAUpdate, _inner, _kv, _mask, _matching, _raise_numeric,
                  _raise_update)

__all__ = ["ShardedWCAState", "head_shard", "exchange_row_sums", "agree_status", "shard_budget"]


def head_shard(heads_total: int, world: int, rank: int) -> slice:
    """The contiguous KV heads of ``rank`` when ``heads_total`` heads are split
    evenly over ``world`` ranks (the C5 layout: 8 KV heads -> 1 per GPU)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    if heads_total < world or heads_total % world:
        raise ValueError("heads_total must be a positive multiple of the world size")
    per = heads_total // world
    return slice(rank * per, (rank + 1) * per)


def exchange_row_sums(partial: Tensor, group=None) -> Tensor:
    """This rank's partial row sums ``[k, n]`` (float64: deviation, norm and,
    at a gate layer, cosine / heads_total) summed over the group in place:
    afterwards every rank holds the sums over all heads (wca.py:55-112)."""
    if partial.dtype != torch.float64 or partial.ndim != 2:
        raise ValueError("row sums must be a float64 [k, n] tensor")
    if _single(group):  # one process holds every head: its sums are complete
        return partial
    dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=group)
    return partial


def _single(group) -> bool:
    return group is None and not (dist.is_available() and dist.is_initialized())


def agree_status(bits: int, device, group=None) -> int:
    """The union (bitwise max) of every rank's status bits, so that every rank
    raises the same error or none does before anything is committed."""
    if _single(group):
        return int(bits)
    flag = torch.tensor([int(bits)], dtype=torch.int32, device=device)
    dist.all_reduce(flag, op=dist.ReduceOp.MAX, group=group)
    return int(flag.item())


def shard_budget(fraction: float, reused_count: int, candidate_count: int) -> int:
    """The selection budget every rank derives from the complete counts
    (wca.py:152-191): min(ceil(fraction * |reused|), |candidates|)."""
    return min(math.ceil(fraction * int(reused_count)), int(candidate_count))


def _row_sums(cached: Tensor, rows: Tensor | None, fresh: Tensor, heads_total: int,
              out: Tensor, with_cosine: bool) -> int:
    """Partial row sums of this rank's heads into out[0] (deviation), out[1]
    (norm) and, with ``with_cosine``, out[2] (cosine / heads_total)."""
    device = cached.device
    c, f = _inner(cached), _inner(fresh)
    n = f.shape[0]
    status = N.Status(device)
    N.check(
        N.load().cs_wca_row_sums(
            c.data_ptr(), c.stride(0), c.stride(1), N.ptr(rows), f.data_ptr(), f.stride(0),
            f.stride(1), n, c.shape[1], c.shape[2], N.DTYPES[c.dtype], int(heads_total),
            out[0].data_ptr(), out[1].data_ptr(), out[2].data_ptr() if with_cosine else None,
            status.ptr, N.stream_of(device),
        ),
        "cs_wca_row_sums",
    )
    return status.read()


class ShardedWCAState(WCAState):
    """``WCAState`` for one rank of a KV-head tensor-parallel group: K/V
    arguments hold this rank's heads only; every rank must call
    ``initialize`` and each ``update`` in the same order (they all-reduce)."""

    group = None
    heads_total: int = 0

    @classmethod
    def initialize(
        cls,
        cached_k: Tensor,
        recomputed_k: Tensor,
        reused_mask: Tensor,
        mandatory_mask: Tensor,
        config: WCAConfig | None = None,
        *,
        heads_total: int,
        group=None,
    ) -> ShardedWCAState:
        config = as_config(config)
        _kv("cached_k", cached_k)
        _matching("recomputed_k", recomputed_k, cached_k)
        if heads_total < cached_k.shape[1]:
            raise ValueError("heads_total must count at least this rank's heads")
        n = cached_k.shape[0]
        device = N.require_cuda(cached_k)
        _mask("reused_mask", reused_mask, n, cached_k.device)
        _mask("mandatory_mask", mandatory_mask, n, cached_k.device)
        if bool(((~reused_mask) & (~mandatory_mask)).any()):
            raise ValueError("every dynamic/non-reused token must be mandatory")
        sums = torch.empty(2, n, dtype=torch.float64, device=device)
        bits = _row_sums(cached_k, None, recomputed_k, heads_total, sums, False)
        exchange_row_sums(sums, group)
        dev, nrm = sums[0], sums[1]
        reused = reused_mask.clone()
        alpha = torch.empty(n, dtype=torch.float64, device=device)
        candidate = torch.empty(n, dtype=torch.bool, device=device)
        counts = torch.empty(2, dtype=torch.int64, device=device)
        status = N.Status(device)
        N.check(
            N.load().cs_wca_weights(
                dev.data_ptr(), nrm.data_ptr(), n, float(config.epsilon),
                int(config.clamp_alpha), reused.data_ptr(), alpha.data_ptr(),
                candidate.data_ptr(), counts.data_ptr(), status.ptr, N.stream_of(device),
            ),
            "cs_wca_weights",
        )
        # the nonfinite decision is the same on every rank (complete sums), or
        # comes from a rank's own inputs: agree on it before raising
        _raise_numeric(agree_status(bits | status.read(), device, group),
                       "squared deviation overflowed float64")
        reused_count, candidate_count = counts.tolist()
        budget = shard_budget(config.correction_fraction, reused_count, candidate_count)
        state = cls(
            config=config,
            reused_mask=reused,
            mandatory_mask=mandatory_mask.clone(),
            initial_deviation=dev.clone(),
            candidate_mask=candidate,
            selected_mask=torch.zeros(n, dtype=torch.bool, device=device),
            removed_mask=torch.zeros(n, dtype=torch.bool, device=device),
            alpha=alpha,
            budget=budget,
        )
        state.group = group
        state.heads_total = int(heads_total)
        state._promote()
        return state

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
        """``WCAState.update`` for this rank's heads, with the weights and the
        gate cosine taken from the all-reduced row sums of every head."""
        indices, ck, cv, fk, fv = self._check_update(
            layer_index, cached_k, cached_v, recomputed_k, recomputed_v, computed_indices)
        device = ck.device
        a = indices.numel()
        gate = layer_index % self.config.gate_interval == 0
        sums = torch.empty(3 if gate else 2, a, dtype=torch.float64, device=device)
        bits = _row_sums(ck, indices, fk, self.heads_total, sums, gate) if a else 0
        exchange_row_sums(sums, self.group)
        next_alpha = torch.empty(a, dtype=torch.float64, device=device)
        status = N.Status(device)
        N.check(
            N.load().cs_wca_weights(
                sums[0].data_ptr(), sums[1].data_ptr(), a, float(self.config.epsilon),
                int(self.config.clamp_alpha), None, next_alpha.data_ptr(), None, None,
                status.ptr, N.stream_of(device),
            ),
            "cs_wca_weights",
        )
        cosine = sums[2] if gate else None
        # the blend weights: the stored ones, or (same_layer) this layer's
        # complete weights at the active rows, without committing them yet
        alpha = self.alpha
        if self.config.weight_update == "same_layer":
            alpha = self.alpha.index_copy(0, indices, next_alpha)
        fused_k, fused_v, _, used, blend_bits = self._blend(
            indices, ck, cv, fk, fv, same_layer=False, cosine=None, paged=paged, alpha=alpha,
            check=False)
        # every rank raises, or none does (the update is all-or-nothing on
        # every rank): agree on the status bits before committing
        _raise_update(agree_status(bits | status.read() | blend_bits, device, self.group))
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

