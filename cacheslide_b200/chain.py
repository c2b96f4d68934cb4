"""Reuse layers chained on the device's own active rows.

In the reference runtime each layer's rows come from the previous layer's WCA
commit: ``active = state.wca.active_indices`` (runtime.py:410), a host tensor,
and the association rows of runtime.py:448-454.  ``ChainedLayers`` runs a
request's layers after the first with that decision left on the device.
``cs_wca_active_rows`` writes the rows, their association flags and their
count.  The WCA update, the CCPE attention and the commit then read the count
from device memory (``a_dev`` / ``nq_dev``), every launch sized by a capacity
(the active rows of layer 1 plus a margin for promotions).  No host read
happens between layers.  ``device=False`` runs the same layers with the
count read back to the host before each layer, the reference's own order,
for comparison.

Inputs are synthetic: per layer, fresh K/V and queries for every token (the
rows a layer computes are gathered from them on the device), the request's
snapshot as the cached K/V, and its paged cache as the arena.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as N
from .reuse import ReuseStep, SyntheticWorkload


class ChainedLayers:
    """Layers 2..L of request ``index`` of a built ``ReuseStep``'s workload."""

    def __init__(self, step: ReuseStep, layers: int, index: int = 0, margin: int = 128,
                 seed: int = 17, gate_interval: int = 2):
        self.step = step
        self.work: SyntheticWorkload = step.work
        self.r = self.work.requests[index]
        self.layers = layers
        self.gate_interval = gate_interval
        cfg = self.work.cfg
        dev = self.work.device
        n, hkv, hq, d = cfg.seq, cfg.kv_heads, cfg.q_heads, cfg.head_dim
        self.cap = self.r.a + margin
        g = torch.Generator().manual_seed(seed)
        r = self.r
        self.fresh_k, self.fresh_v, self.q = [], [], []
        for _ in range(layers):
            self.fresh_k.append((r.cached_k.float().cpu() + 0.05 * torch.randn(
                n, hkv, d, generator=g)).to(cfg.dtype).to(dev))
            self.fresh_v.append((r.cached_v.float().cpu() + 0.05 * torch.randn(
                n, hkv, d, generator=g)).to(cfg.dtype).to(dev))
            self.q.append((torch.randn(n, hq, d, generator=g) / d ** 0.5).to(cfg.dtype).to(dev))
        cap = self.cap
        self.rows = torch.empty(cap, dtype=torch.int64, device=dev)
        self.assoc = torch.empty(cap, dtype=torch.uint8, device=dev)
        self.count = torch.empty(1, dtype=torch.int64, device=dev)
        self.next_alpha = torch.empty(cap, dtype=torch.float64, device=dev)
        self.used = torch.empty_like(self.next_alpha)
        self.cos = torch.empty_like(self.next_alpha)
        self.out = torch.empty(cap, hq, d, dtype=cfg.dtype, device=dev)
        self.removed_list = torch.empty(n, dtype=torch.int64, device=dev)
        self.promoted = torch.empty(n, dtype=torch.int64, device=dev)
        self.counts = torch.zeros(2, dtype=torch.int64, device=dev)
        self.lib = N.load()

    def layer(self, layer: int, device: bool = True) -> None:
        """Layer ``layer`` (1-based, >= 2) on the rows the previous commit chose.

        Everything runs on torch's current stream: the row gathers are torch
        ops, and their buffers are released to torch's allocator after the
        layer's launches are queued, which is safe only in one stream order.
        """
        cfg, r, lib, step = self.work.cfg, self.r, self.lib, self.step
        s = N.stream_of(self.work.device)
        n, cap = cfg.seq, self.cap
        st = r.status_ptr
        N.check(lib.cs_wca_active_rows(r.selected.data_ptr(), r.mandatory.data_ptr(), n, cap,
                                       self.rows.data_ptr(), self.assoc.data_ptr(),
                                       self.count.data_ptr(), st, s), "cs_wca_active_rows")
        if device:
            a, a_dev = cap, self.count.data_ptr()
        else:
            torch.cuda.synchronize(self.work.device)
            a, a_dev = int(self.count.item()), None
        li = layer - 1
        idx = self.rows[:a].clamp_min(0)
        fk = self.fresh_k[li].index_select(0, idx)
        fv = self.fresh_v[li].index_select(0, idx)
        slots = r.slots.index_select(0, idx)
        gate = layer % self.gate_interval == 0
        upd = (N.UpdateItem * 1)(N.UpdateItem(
            r.cached_k.data_ptr(), r.cached_v.data_ptr(), r.cached_k.stride(0),
            r.cached_k.stride(1), fk.data_ptr(), fv.data_ptr(), fk.stride(0), fk.stride(1),
            self.rows.data_ptr(), a, r.alpha.data_ptr(), r.mandatory.data_ptr(), None, None,
            self.next_alpha.data_ptr(), self.used.data_ptr(),
            self.cos.data_ptr() if gate else None, slots.data_ptr(), st, a_dev))
        N.check(lib.cs_wca_update_batch(upd, 1, cfg.kv_heads, cfg.head_dim, N.DTYPES[cfg.dtype],
                                        0, 1e-8, 0, ctypes.byref(step.kv), s), "update")
        q = self.q[li].index_select(0, idx)
        co = r.offsets.index_select(1, idx).contiguous()
        p = step._attn_params(r)
        p.q = q.data_ptr()
        p.q_stride_tok, p.q_stride_head = q.stride(0), q.stride(1)
        p.nq, p.nq_dev = a, a_dev
        p.qpos = self.rows.data_ptr()
        p.q_selected = self.assoc.data_ptr()
        p.chunk_off = co.data_ptr()
        p.co_stride_h, p.co_stride_q = co.stride(0), co.stride(1)
        p.out = self.out.data_ptr()
        p.o_stride_tok, p.o_stride_head = self.out.stride(0), self.out.stride(1)
        N.check(lib.cs_cope_attn_prefill(ctypes.byref(p), s), "prefill")
        com = (N.CommitItem * 1)(N.CommitItem(
            self.rows.data_ptr(), a, self.next_alpha.data_ptr(),
            self.cos.data_ptr() if gate else None, n, r.budget, r.dev.data_ptr(),
            r.alpha.data_ptr(), r.candidate.data_ptr(), r.selected.data_ptr(),
            r.removed.data_ptr(), self.removed_list.data_ptr(), self.promoted.data_ptr(),
            self.counts.data_ptr(), st, a_dev))
        N.check(lib.cs_wca_commit_batch(com, 1, 0.12, 0, s), "commit")
        # the gathered inputs stay referenced until the next layer's are made;
        # freed then, their memory is reused only by work queued after these
        # launches on the same stream
        self._keep = (fk, fv, slots, q, co, upd, com)

    def run(self, device: bool = True) -> None:
        """Layers 2..L back to back on torch's current stream."""
        for layer in range(2, self.layers + 1):
            self.layer(layer, device)
