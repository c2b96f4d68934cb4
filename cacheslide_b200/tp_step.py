"""One reuse-prefill layer of a KV-head tensor-parallel rank (the C5 layout).

Llama-3-70B at TP8 holds 8 KV heads and 64 query heads; over ``world`` ranks
each rank holds ``8 / world`` KV heads and ``64 / world`` query heads (one
and eight at eight ranks).  A step on one rank, for every request of the
rank's batch (the same requests on every rank, each rank its own heads):

1. SLIDE: the layer's snapshot K/V written into the rank's paged pool
   (``cs_slide_scatter_batch``);
2. WCA with the head sums exchanged: ``tp.ShardedWCAState.initialize`` and
   ``update`` (one float64 all-reduce of the per-shard row sums each, and a
   status agreement), the fused rows blended straight into their paged slots;
3. CCPE attention of the active rows through the slot table, all requests in
   one tensor-core launch (npos 128, chunk-reset positions);
4. ``o_proj``: the rank's attention rows times its row block of the output
   projection (``[active rows, 8192]``, cuBLAS through torch), then one NCCL
   all-reduce (sum) of ``[all requests' active rows, 8192]`` bf16 -- the
   collective that follows attention in a tensor-parallel Llama-3-70B-shaped
   model (8 KV heads split over the ranks).

The token layout (chunks, which chunk is recomputed, reused / mandatory
masks, paged blocks) is the same on every rank; the head data are seeded per
rank.  The WCA decisions come from all-reduced sums, so every rank computes
the same active rows; a first pass at construction fixes them (as
``reuse.ReuseStep`` does) so the attention arguments are built once.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _native as N
from .policy import WCAConfig
from .tp import ShardedWCAState, head_shard


@dataclass(frozen=True)
class TPWorkloadConfig:
    requests: int = 8
    q_heads_total: int = 64
    kv_heads_total: int = 8
    head_dim: int = 128
    seq: int = 65536
    chunks: int = 32
    npos: int = 128
    block: int = 16
    fraction: float = 0.10
    hidden: int = 8192
    seed: int = 0
    dynamic_chunk: int = 13
    profile_noise: float = 0.05
    dtype: torch.dtype = torch.bfloat16


class _Arena:
    """The ``paged=(arena, slots)`` argument of ``WCAState.update``: a pool
    view with ``device_view()``."""

    def __init__(self, view: N.PagedKV):
        self._view = view

    def device_view(self) -> N.PagedKV:
        return self._view


class ShardedReuseStep:
    """One reuse-prefill layer of a tensor-parallel rank (see the module)."""

    def __init__(self, cfg: TPWorkloadConfig, device: torch.device, group=None,
                 rank: int = 0, world: int = 1):
        self.cfg, self.device, self.group = cfg, device, group
        hs = head_shard(cfg.kv_heads_total, world, rank)
        hkv = hs.stop - hs.start
        hq = cfg.q_heads_total // world
        if cfg.q_heads_total % world or hq % hkv:
            raise ValueError("query heads must split evenly over the ranks and KV heads")
        self.hkv, self.hq = hkv, hq
        n, d, bs = cfg.seq, cfg.head_dim, cfg.block
        dt = cfg.dtype
        self.lib = N.load()
        self.wca_config = WCAConfig(correction_fraction=cfg.fraction, gate_interval=1)
        # the layout: identical on every rank
        lay = torch.Generator().manual_seed(cfg.seed)
        clen = n // cfg.chunks
        blocks_per_req = (n + bs - 1) // bs
        total_blocks = blocks_per_req * cfg.requests
        pool = torch.randperm(total_blocks, generator=lay).to(device)
        self.cache = torch.zeros(total_blocks, hkv, bs, 2 * d, dtype=dt, device=device)
        self.kv = N.paged_view(self.cache)
        self.arena = _Arena(self.kv)
        # head data: per rank, generated on the device
        g = torch.Generator(device=device).manual_seed(cfg.seed * 1009 + rank + 1)

        def randn(*shape, scale=1.0):
            return (torch.randn(*shape, generator=g, device=device) * scale).to(dt)

        self.status = torch.zeros(cfg.requests, dtype=torch.int32, device=device)
        self.requests = []
        tok = torch.arange(n, device=device)
        chunk_of = torch.clamp(tok // clen, max=cfg.chunks - 1)
        dyn = cfg.dynamic_chunk % cfg.chunks
        for b in range(cfg.requests):
            r = _Request()
            r.block_table = pool[b * blocks_per_req:(b + 1) * blocks_per_req]
            r.slots = (r.block_table[tok // bs] * bs + tok % bs).contiguous()
            r.key_chunk = chunk_of.to(torch.int32).contiguous()
            r.reused = (chunk_of != dyn).contiguous()
            r.mandatory = ~r.reused
            r.mandatory[n - 1] = True
            r.cached_k = randn(n, hkv, d, scale=1 / math.sqrt(d))
            r.cached_v = randn(n, hkv, d)
            r.calib_k = (r.cached_k.float() + cfg.profile_noise * torch.randn(
                n, hkv, d, generator=g, device=device)).to(dt)
            r.calib_k[r.mandatory] = r.cached_k[r.mandatory]
            r.fresh_k = (r.cached_k.float() + cfg.profile_noise * torch.randn(
                n, hkv, d, generator=g, device=device)).to(dt)
            r.fresh_v = (r.cached_v.float() + cfg.profile_noise * torch.randn(
                n, hkv, d, generator=g, device=device)).to(dt)
            r.status_ptr = self.status[b:b + 1].data_ptr()
            self.requests.append(r)
        self.E = (torch.randn(d, cfg.npos, generator=g, device=device) * 0.02).contiguous()
        # the row block of o_proj this rank holds: [hq * d, hidden]
        self.w_o = randn(hq * d, cfg.hidden, scale=1 / math.sqrt(cfg.q_heads_total * d))
        # first pass: the WCA decisions (the same on every rank), active rows
        self.scatter_items = (N.ScatterItem * len(self.requests))(*[N.ScatterItem(
            r.slots.data_ptr(), None, n, r.cached_k.data_ptr(), r.cached_v.data_ptr(),
            r.cached_k.stride(0), r.cached_k.stride(1), r.status_ptr) for r in self.requests])
        self._scatter(N.stream_of(device))
        for r in self.requests:
            st = ShardedWCAState.initialize(r.cached_k, r.calib_k, r.reused, r.mandatory,
                                            self.wca_config, heads_total=cfg.kv_heads_total,
                                            group=group)
            r.active = st.active_indices
            r.a = r.active.numel()
            r.q = randn(r.a, hq, d, scale=1 / math.sqrt(d))
            r.out = torch.empty(r.a, hq, d, dtype=dt, device=device)
            # chunk-reset offsets of the active rows: the canonical count
            # entering each older chunk (an average gate of 0.5 a key, with
            # jitter); the query's own and newer chunks and dynamic rows carry
            pos = r.active.float()
            ends = (torch.arange(cfg.chunks, device=device, dtype=torch.float32) + 1) * clen - 1
            off = 0.5 * (pos[:, None] - ends[None, :])
            jitter = 1 + 0.05 * torch.randn(hq, r.a, cfg.chunks, generator=g, device=device)
            off = (off[None] * jitter).clamp_min(0)
            own = torch.arange(cfg.chunks, device=device)[None, :] >= chunk_of[r.active][:, None]
            off[:, own] = -1.0
            off[:, ~r.reused[r.active]] = -1.0
            r.co = off.contiguous()
            r.params = self._attn_params(r)
        self.attn_params = (N.AttnParams * len(self.requests))(
            *[r.params for r in self.requests])
        offs = [0]
        for r in self.requests:
            offs.append(offs[-1] + r.a)
        self.row_offsets = offs
        self.proj = torch.empty(offs[-1], cfg.hidden, dtype=dt, device=device)
        torch.cuda.synchronize(device)

    def _attn_params(self, r) -> N.AttnParams:
        c = self.cfg
        p = N.AttnParams()
        p.q = r.q.data_ptr()
        p.q_stride_tok, p.q_stride_head = r.q.stride(0), r.q.stride(1)
        p.nq, p.hq, p.d = r.a, self.hq, c.head_dim
        p.qpos = r.active.data_ptr()
        p.paged = self.kv
        p.kv_slots = r.slots.data_ptr()
        p.nk, p.hkv, p.dv = c.seq, self.hkv, c.head_dim
        p.E = self.E.data_ptr()
        p.e_stride_d, p.e_stride_p = self.E.stride()
        p.npos = c.npos
        p.scale = math.sqrt(c.head_dim)
        p.pos_mode = N.POS_CHUNK
        p.key_chunk = r.key_chunk.data_ptr()
        p.chunk_off = r.co.data_ptr()
        p.co_stride_h, p.co_stride_q = r.co.stride(0), r.co.stride(1)
        p.nchunks = c.chunks
        p.atol = 1e-6
        p.out = r.out.data_ptr()
        p.o_stride_tok, p.o_stride_head = r.out.stride(0), r.out.stride(1)
        p.in_dtype = p.out_dtype = N.DTYPES[c.dtype]
        p.status = r.status_ptr
        return p

    def _scatter(self, stream) -> None:
        N.check(self.lib.cs_slide_scatter_batch(ctypes.byref(self.kv), self.scatter_items,
                                                len(self.scatter_items), stream),
                "cs_slide_scatter_batch")

    def wca(self) -> None:
        """WCA of every request with the head sums all-reduced: initialize,
        then the layer's update with the fused rows written to their slots."""
        for r in self.requests:
            st = ShardedWCAState.initialize(r.cached_k, r.calib_k, r.reused, r.mandatory,
                                            self.wca_config, heads_total=self.cfg.kv_heads_total,
                                            group=self.group)
            idx = st.active_indices
            st.update(2, r.cached_k, r.cached_v, r.fresh_k.index_select(0, idx),
                      r.fresh_v.index_select(0, idx), idx,
                      paged=(self.arena, r.slots.index_select(0, idx)))

    def attention(self, stream) -> None:
        N.check(self.lib.cs_cope_attn_prefill_batch(self.attn_params, len(self.requests),
                                                    stream), "cs_cope_attn_prefill_batch")

    def o_proj(self) -> None:
        """Each request's attention rows times the rank's o_proj rows, into
        its slice of the all-reduce buffer."""
        for r, lo, hi in zip(self.requests, self.row_offsets, self.row_offsets[1:]):
            torch.matmul(r.out.view(r.a, -1), self.w_o, out=self.proj[lo:hi])

    def all_reduce(self) -> None:
        if self.group is not None or (dist.is_initialized() and dist.get_world_size() > 1):
            dist.all_reduce(self.proj, op=dist.ReduceOp.SUM, group=self.group)

    def run(self, stream, marks=None) -> None:
        """One step on ``stream`` (a torch stream, current for the torch ops);
        ``marks`` (five CUDA events) split it into SLIDE, WCA, attention,
        o_proj and the all-reduce."""
        s = stream.cuda_stream

        def mark(i):
            if marks is not None:
                marks[i].record(stream)

        mark(0)
        self._scatter(s)
        mark(1)
        self.wca()
        mark(2)
        self.attention(s)
        mark(3)
        self.o_proj()
        mark(4)
        self.all_reduce()
        mark(5)

    def check_status(self) -> None:
        acc = 0
        for word in self.status.cpu().tolist():
            acc |= int(word)
        if acc:
            raise RuntimeError(f"device status bits set: {acc:#x}")

    def attention_flops(self) -> float:
        """QK over every causal cell, PV over every causal cell (no
        association policy here), and q.E, of all requests."""
        c = self.cfg
        total = 0.0
        for r in self.requests:
            causal = float((r.active + 1).sum())
            total += 4 * c.head_dim * self.hq * causal
            total += 2 * r.a * self.hq * c.npos * c.head_dim
        return total


class _Request:
    """Device tensors of one request on one rank."""
