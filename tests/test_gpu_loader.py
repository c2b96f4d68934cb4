"""The layer-pipelined snapshot loader (``loader.SnapshotLoader``): pinned
host snapshots of several layers copied on the loader's stream and
scattered into each layer's paged slots, consumed by a compute stream that
waits on each layer's event; bit-exact pool contents, and the reference's
non-finite snapshot rejection (runtime.py:192-229)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from cacheslide_b200 import _native as N
from cacheslide_b200.loader import SnapshotLoader

pytestmark = pytest.mark.gpu


def test_layers_land_in_their_slots_in_order(cuda):
    g = torch.Generator().manual_seed(4)
    layers, nb, hkv, bs, d, n = 5, 64, 4, 16, 128, 700
    pools = [torch.zeros(nb, hkv, bs, 2 * d, dtype=torch.bfloat16, device=cuda)
             for _ in range(layers)]
    perm = torch.randperm(nb * bs, generator=g)[:n].to(cuda)
    snaps = [(torch.randn(n, hkv, d, generator=g).to(torch.bfloat16).pin_memory(),
              torch.randn(n, hkv, d, generator=g).to(torch.bfloat16).pin_memory())
             for _ in range(layers)]
    torch.cuda.synchronize()  # pools and slots ready before the loader's stream starts
    loader = SnapshotLoader(cuda, depth=2)
    compute = torch.cuda.Stream(device=cuda)
    loads = [loader.submit(0, *snaps[0], N.paged_view(pools[0]), perm)]
    sums = []
    for layer in range(layers):
        if layer + 1 < layers:  # the next layer copies while this one computes
            loads.append(loader.submit(layer + 1, *snaps[layer + 1],
                                       N.paged_view(pools[layer + 1]), perm))
        loads[layer].wait(compute)
        with torch.cuda.stream(compute):
            sums.append(pools[layer].float().sum())
    torch.cuda.synchronize()
    for layer, (k, v) in enumerate(snaps):
        loads[layer].result()
        pool = pools[layer]
        got_k = pool[perm // bs, :, perm % bs, :d].cpu()
        got_v = pool[perm // bs, :, perm % bs, d:].cpu()
        assert torch.equal(got_k.view(torch.int16), k.view(torch.int16))
        assert torch.equal(got_v.view(torch.int16), v.view(torch.int16))
        want = float(k.float().sum() + v.float().sum())
        np.testing.assert_allclose(float(sums[layer]), want, rtol=1e-3)


def test_nonfinite_snapshot_is_rejected(cuda):
    pool = torch.zeros(8, 2, 16, 128, dtype=torch.float16, device=cuda)
    k = torch.randn(10, 2, 64).to(torch.float16)
    v = torch.randn(10, 2, 64).to(torch.float16)
    v[3, 1, 7] = float("nan")
    slots = torch.arange(10, dtype=torch.int64, device=cuda)
    torch.cuda.synchronize()
    load = SnapshotLoader(cuda).submit(0, k.pin_memory(), v.pin_memory(), N.paged_view(pool),
                                       slots)
    with pytest.raises(ValueError, match="nonfinite"):
        load.result()
    with pytest.raises(ValueError, match="geometry"):
        SnapshotLoader(cuda).submit(0, k[:, :1], v[:, :1], N.paged_view(pool), slots)
