"""Multi-rank paths on CPU: world_size-2 `gloo` process groups.

* KV-head tensor parallelism of WCA (``cacheslide_b200.tp``): the head
  shards' partial row sums (deviation, norm, cosine / heads_total), summed by
  ``tp.exchange_row_sums``, reproduce the full-head reductions of the
  reference (``wca.py:55-112``), so every rank selects, removes and promotes
  the same tokens as an unsharded state.  The partial sums are the host
  values ``cs_wca_row_sums`` computes on the device (each rank's heads); the
  exchange, the budget (``tp.shard_budget``) and the status agreement
  (``tp.agree_status``) are ``tp.py``'s own functions, run over gloo.
* Request sharding (``bench.py --gpus N``): ranks build independent request
  sets from per-rank seeds and the job time is the maximum over ranks.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cacheslide_b200.tp import agree_status, exchange_row_sums, head_shard, shard_budget
from oracle import wca as owca

WORLD = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(fn, *args):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_entry, args=(r, port, fn, args)) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    for p in procs:
        if p.is_alive():
            p.kill()
            pytest.fail("a rank did not finish")
        assert p.exitcode == 0, f"rank failed with exit code {p.exitcode}"


def _entry(rank, port, fn, args):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=60))
    try:
        fn(rank, *args)
    finally:
        dist.destroy_process_group()


def _exchange(parts: list[np.ndarray]) -> np.ndarray:
    """This rank's partial row sums through ``tp.exchange_row_sums``."""
    t = torch.from_numpy(np.ascontiguousarray(np.stack(parts), dtype=np.float64))
    out = exchange_row_sums(t)
    assert out is t  # summed in place, as the device path relies on
    return t.numpy()


class ShardedOracleWCA(owca.OracleWCA):
    """The decisions of ``ShardedWCAState`` on host inputs: this rank's heads
    only, partial row sums exchanged by ``tp.exchange_row_sums`` before any
    decision, the budget from ``tp.shard_budget``."""

    def initialize(self, cached, fresh, reused, mandatory, heads_total):
        self.heads_total = heads_total
        c64, f64 = cached.astype(np.float64), fresh.astype(np.float64)
        dev, nrm = _exchange([np.square(f64 - c64).sum((1, 2)), np.square(c64).sum((1, 2))])
        self.reused, self.mandatory = reused.copy(), mandatory.copy()
        self.initial = dev.copy()
        self.candidate = reused & (dev > 0)
        self.budget = shard_budget(self.correction_fraction, int(reused.sum()),
                                   int(self.candidate.sum()))
        self.selected = np.zeros_like(self.candidate)
        self.removed = np.zeros_like(self.candidate)
        self.alpha = dev / (nrm + self.epsilon)
        self.last_layer = 1
        self._promote()
        return self

    def update(self, layer, cached_k, cached_v, fresh_k, fresh_v):
        idx = self.active
        old_k, old_v = cached_k[idx], cached_v[idx]
        o64, f64 = old_k.astype(np.float64), fresh_k.astype(np.float64)
        gate = layer % self.gate_interval == 0
        parts = [np.square(f64 - o64).sum((1, 2)), np.square(o64).sum((1, 2))]
        if gate:
            heads = fresh_k.shape[1]
            parts.append(owca.mean_head_cosine(fresh_k, old_k, self.epsilon) * heads
                         / self.heads_total)
        sums = _exchange(parts)
        nxt = sums[0] / (sums[1] + self.epsilon)
        used = self.alpha[idx] if self.weight_update == "previous_layer" else nxt
        used = np.where(self.mandatory[idx], 1.0, used)
        w = used[:, None, None]
        fk = w * f64 + (1 - w) * o64
        fv = w * fresh_v.astype(np.float64) + (1 - w) * old_v.astype(np.float64)
        removed = idx[:0]
        if gate:
            cos = sums[2]
            metric = cos if self.convergence_mode == "paper_cosine_lt" else 1 - cos
            removed = idx[self.selected[idx] & (metric < self.convergence_threshold)]
        self.alpha[idx] = nxt
        self.selected[removed] = False
        self.candidate[removed] = False
        self.removed[removed] = True
        promoted = self._promote()
        self.last_layer = layer
        return dict(indices=idx, fused_k=fk, fused_v=fv, alpha=used, removed=removed,
                    promoted=promoted, next_indices=self.active)


def _tp_ranks(rank, weight_update):
    heads, n, d = 8, 384, 16
    rng = np.random.default_rng(11)
    mandatory = np.zeros(n, bool)
    mandatory[-40:] = True
    reused = ~mandatory
    cached = rng.standard_normal((n, heads, d)).astype(np.float32)
    fresh = cached + rng.standard_normal((n, heads, d)).astype(np.float32) * 0.3
    hs = head_shard(heads, WORLD, rank)
    cfg = dict(correction_fraction=0.2, weight_update=weight_update, gate_interval=2)
    full = owca.OracleWCA(**cfg).initialize(cached, fresh, reused, mandatory)
    part = ShardedOracleWCA(**cfg).initialize(cached[:, hs], fresh[:, hs], reused, mandatory,
                                              heads)
    np.testing.assert_array_equal(part.selected, full.selected)
    np.testing.assert_allclose(part.alpha, full.alpha, rtol=1e-12)
    removed_total = 0
    for layer in range(2, 7):
        ck = rng.standard_normal((n, heads, d)).astype(np.float32)
        cv = rng.standard_normal((n, heads, d)).astype(np.float32)
        a = len(full.active)
        rk = ck[full.active] + rng.standard_normal((a, heads, d)).astype(np.float32) * 0.2
        far = rng.random(a) < 0.3  # rows whose recomputation disagrees: gate removals
        rk[far] = rng.standard_normal((int(far.sum()), heads, d)).astype(np.float32)
        rv = cv[full.active] + rng.standard_normal((a, heads, d)).astype(np.float32) * 0.2
        want = full.update(layer, ck, cv, rk, rv)
        got = part.update(layer, ck[:, hs], cv[:, hs], rk[:, hs], rv[:, hs])
        for key in ("indices", "removed", "promoted", "next_indices"):
            np.testing.assert_array_equal(got[key], want[key], err_msg=key)
        # weights from differently ordered float64 sums: equal to rounding
        np.testing.assert_allclose(got["alpha"], want["alpha"], rtol=1e-12)
        np.testing.assert_allclose(got["fused_k"], want["fused_k"][:, hs], rtol=1e-9, atol=1e-12)
        np.testing.assert_allclose(got["fused_v"], want["fused_v"][:, hs], rtol=1e-9, atol=1e-12)
        removed_total += len(want["removed"])
    assert removed_total > 0  # the gate path was exercised


@pytest.mark.parametrize("weight_update", ["previous_layer", "same_layer"])
def test_head_sharded_wca_selects_like_the_full_state(weight_update):
    _run(_tp_ranks, weight_update)


def _agreement_ranks(rank):
    cpu = torch.device("cpu")
    # a status bit raised on one rank only reaches every rank
    assert agree_status(0x4 if rank == 1 else 0, cpu) == 0x4
    assert agree_status(0x1 if rank == 0 else 0x2, cpu) == 0x2  # max, as the device flags
    assert agree_status(0, cpu) == 0
    # partial sums of disjoint head shards add up to the full-head sums
    part = torch.full((3, 5), float(rank + 1), dtype=torch.float64)
    exchange_row_sums(part)
    assert torch.equal(part, torch.full((3, 5), 3.0, dtype=torch.float64))
    # a malformed buffer is rejected on every rank before any collective
    for bad in (torch.zeros(2, 4, dtype=torch.float32), torch.zeros(4, dtype=torch.float64)):
        with pytest.raises(ValueError):
            exchange_row_sums(bad)
    # the ranks are still in step: one more collective completes
    assert agree_status(rank, cpu) == WORLD - 1


def test_status_agreement_and_row_sum_exchange_over_gloo():
    _run(_agreement_ranks)


def test_shard_budget_follows_the_reference_rounding():
    assert shard_budget(0.15, 3584, 3584) == 538  # C2: ceil(0.15 * 3584)
    assert shard_budget(0.2, 10, 1) == 1           # capped by the candidates
    assert shard_budget(0.0, 10, 10) == 0
    assert shard_budget(1.0, 7, 9) == 7


def test_head_shard_splits_evenly_and_rejects_bad_layouts():
    assert [head_shard(8, 8, r) for r in (0, 7)] == [slice(0, 1), slice(7, 8)]
    assert head_shard(8, 2, 1) == slice(4, 8)
    for bad in ((8, 3, 0), (4, 8, 0), (8, 2, 2), (8, 0, 0)):
        with pytest.raises(ValueError):
            head_shard(*bad)


def _request_ranks(rank):
    from cacheslide_b200.reuse import SyntheticWorkload, WorkloadConfig

    cfg = WorkloadConfig(requests=1, seq=1024, seed=1000 + rank)  # bench.py's per-rank seed
    work = SyntheticWorkload(cfg, torch.device("cpu"))
    q = work.requests[0].cached_k.float()
    sums = torch.zeros(WORLD, dtype=torch.float64)
    sums[rank] = float(q.abs().sum())
    dist.all_reduce(sums)
    assert sums[0] != sums[1]  # independent requests on the two ranks
    ms = torch.tensor([10.0 + 5.0 * rank], dtype=torch.float64)  # a rank's device time
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    assert float(ms) == 15.0  # the job time is the slowest rank's


def test_request_sharded_ranks_are_independent_and_time_the_slowest():
    _run(_request_ranks)
