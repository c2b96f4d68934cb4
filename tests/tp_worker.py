"""One rank of the 2-GPU KV-head tensor-parallel WCA check (launched by
tests/test_gpu_tp.py through torch.distributed.run, NCCL).

Every rank holds the full seeded K/V of 8 KV heads, runs the unsharded
``WCAState`` on them as the reference, and ``ShardedWCAState`` on its own
heads only; the two must select, remove and promote the same tokens and fuse
the rank's heads alike, in both weight orders.
"""

from __future__ import annotations

import datetime
import math
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from cacheslide_b200.policy import WCAConfig  # noqa: E402
from cacheslide_b200.tp import ShardedWCAState, head_shard  # noqa: E402
from cacheslide_b200.wca import WCAState  # noqa: E402


def run(rank: int, world: int, dev: torch.device, mode: str) -> int:
    g = torch.Generator().manual_seed(11)
    heads, n, d = 8, 2048, 128
    bf = torch.bfloat16

    def randn(*shape):
        return torch.randn(*shape, generator=g)

    cached = (randn(n, heads, d) / math.sqrt(d)).to(bf).to(dev)
    fresh = (cached.float().cpu() + 0.3 * randn(n, heads, d) / math.sqrt(d)).to(bf).to(dev)
    mandatory = torch.zeros(n, dtype=torch.bool)
    mandatory[-64:] = True
    reused = (~mandatory).to(dev)
    mandatory = mandatory.to(dev)
    hs = head_shard(heads, world, rank)
    cfg = WCAConfig(correction_fraction=0.2, weight_update=mode, gate_interval=2)
    full = WCAState.initialize(cached, fresh, reused, mandatory, cfg)
    part = ShardedWCAState.initialize(cached[:, hs], fresh[:, hs], reused, mandatory, cfg,
                                      heads_total=heads)
    assert torch.equal(part.selected_mask, full.selected_mask), "initial selection"
    torch.testing.assert_close(part.alpha, full.alpha, rtol=1e-12, atol=0)
    removed = 0
    for layer in range(2, 7):
        ck = (randn(n, heads, d) / math.sqrt(d)).to(bf).to(dev)
        cv = randn(n, heads, d).to(bf).to(dev)
        idx = full.active_indices
        a = idx.numel()
        rk = ck[idx].float().cpu() + 0.2 * randn(a, heads, d) / math.sqrt(d)
        far = torch.rand(a, generator=g) < 0.3  # disagreeing rows: gate removals
        rk[far] = randn(int(far.sum()), heads, d) / math.sqrt(d)
        rk = rk.to(bf).to(dev)
        rv = (cv[idx].float().cpu() + 0.2 * randn(a, heads, d)).to(bf).to(dev)
        want = full.update(layer, ck, cv, rk, rv)
        got = part.update(layer, ck[:, hs], cv[:, hs], rk[:, hs], rv[:, hs])
        for key in ("indices", "removed_indices", "promoted_indices", "next_indices"):
            assert torch.equal(getattr(got, key), getattr(want, key)), f"layer {layer}: {key}"
        # weights from differently ordered float64 sums: equal to rounding
        torch.testing.assert_close(got.alpha, want.alpha, rtol=1e-12, atol=0)
        for name in ("fused_k", "fused_v"):
            torch.testing.assert_close(getattr(got, name).float(),
                                       getattr(want, name)[:, hs].float(), rtol=1e-2, atol=1e-2)
        removed += want.removed_indices.numel()
    assert removed > 0, "the gate path was not exercised"
    return removed


def main() -> None:
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        for mode in ("previous_layer", "same_layer"):
            removed = run(rank, world, dev, mode)
            if rank == 0:
                print(f"{mode}: selections agree across {world} ranks ({removed} gate removals)")
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
