"""The selective layer loop's QKV projection on the tensor cores
(``cs_qkv_gather_lora`` through ``layer.selective_qkv``): rows gathered from
the previous layer's output or the layer's snapshot (runtime.py:409-460),
projected with the LoRA delta in the same accumulator (artifacts.py:189-193),
against a float32 torch computation of the reference's steps (index copies,
``F.linear(h, W)`` + ``F.linear(F.linear(h, A), B)`` with the inner product
rounded to the input dtype as a 16-bit model does)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from cacheslide_b200.layer import row_sources, selective_qkv

pytestmark = pytest.mark.gpu


def _reference(prev_h, previous, snap_h, fixed, active, n, w, la, lb):
    lookup = torch.full((n,), -1, dtype=torch.long, device=w.device)
    lookup[previous] = torch.arange(previous.numel(), device=w.device)
    ordinal = torch.full((n,), -1, dtype=torch.long, device=w.device)
    ordinal[fixed] = torch.arange(fixed.numel(), device=w.device)
    rows = lookup[active]
    cont = rows >= 0
    h = prev_h.new_empty((active.numel(), prev_h.shape[1]))
    h[cont] = prev_h[rows[cont]]
    h[~cont] = snap_h[ordinal[active[~cont]]]
    out = F.linear(h.float(), w.float())
    if la is not None:
        t = F.linear(h.float(), la.float()).to(w.dtype).float()
        out = out + F.linear(t, lb.float())
    return out


@pytest.mark.parametrize("n,hidden,n_out,rank,dtype", [
    (700, 512, 768, 16, torch.bfloat16),
    (300, 1024, 512, 0, torch.bfloat16),
    (1500, 256, 256, 24, torch.float16),
    (90, 4096, 6144, 16, torch.bfloat16),   # the Mistral-7B QKV shape, a short prompt
])
def test_selective_qkv_matches_the_reference_steps(cuda, n, hidden, n_out, rank, dtype):
    g = torch.Generator().manual_seed(n + hidden + rank)
    fixed = torch.sort(torch.randperm(n, generator=g)[: int(0.8 * n)]).values
    previous = torch.sort(torch.randperm(n, generator=g)[: int(0.3 * n)]).values
    dyn = torch.tensor(sorted(set(range(n)) - set(fixed.tolist())), dtype=torch.long)
    # active: every dynamic row (continuing when previous had it) + some fixed rows
    extra = fixed[torch.randperm(fixed.numel(), generator=g)[: int(0.2 * n)]]
    active = torch.unique(torch.cat([dyn, extra, previous]))
    prev_only = previous  # dynamic rows must be in previous to be found
    previous = torch.unique(torch.cat([prev_only, dyn]))
    dev = lambda t: t.to(cuda)  # noqa: E731
    prev_h = dev((torch.randn(previous.numel(), hidden, generator=g)).to(dtype))
    snap_h = dev((torch.randn(fixed.numel(), hidden, generator=g)).to(dtype))
    w = dev((torch.randn(n_out, hidden, generator=g) / hidden ** 0.5).to(dtype))
    la = lb = None
    if rank:
        la = dev((torch.randn(rank, hidden, generator=g) / hidden ** 0.5).to(dtype))
        lb = dev((torch.randn(n_out, rank, generator=g) * 0.5).to(dtype))
    args = (prev_h, dev(previous), snap_h, dev(fixed), dev(active), n)
    got = selective_qkv(*args, w, la, lb)
    want = _reference(*args, w, la, lb)
    torch.testing.assert_close(got.float(), want, atol=3e-2, rtol=2e-2)


def test_lost_dynamic_row_raises(cuda):
    n = 10
    fixed = torch.tensor([0, 1, 2, 3, 4], device=cuda)
    previous = torch.tensor([5, 6], device=cuda)
    with pytest.raises(ValueError, match="mandatory dynamic row was lost"):
        row_sources(previous, torch.tensor([5, 7], device=cuda), fixed, n)
