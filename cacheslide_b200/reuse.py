"""Fused reuse-prefill layer and decode step (the runtime.attention hot path).

Reference call stack (runtime.py:474-609): for one layer of a reuse hit the
runtime writes the cached K/V snapshot into the request's paged arena
(``write_prefill``), fuses the recomputed active rows with WCA
(``WCAState.update`` + ``update_selected``), gathers the whole logical K/V
back into a dense copy and runs ``cope_attention`` with the canonical
position policy and the selected-association policy.  ``ReuseStep`` runs the
same layer as a fixed sequence of CUDA launches per request, with no host
synchronisation and no dense gather; the requests' sequences are independent
and run on one stream each, forked from and joined back into the caller's
stream with events:

1. ``cs_slide_scatter``   baseline snapshot -> canonical paged slots;
2. ``cs_wca_initialize``  deviation / weight / candidates of the calibration
   layer (+ ``cs_wca_commit`` selecting the top budget);
3. ``cs_wca_update``      blend of the active rows written straight into their
   paged slots;
4. ``cs_wca_commit``      weight store, cosine gate, promotion;
5. ``cs_cope_attn_prefill`` CCPE attention of the active rows over all keys,
   read through the slot table (chunk-reset canonical positions and the
   association policy evaluated in-kernel).

``SyntheticWorkload`` builds the seeded inputs of the kernel microbenchmark
(batch of requests, shuffled paged blocks, profile K = K + N(0, 0.05)).
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _native as N


@dataclass(frozen=True)
class WorkloadConfig:
    requests: int = 8
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    seq: int = 4096
    chunks: int = 8
    npos: int = 64
    block: int = 16
    fraction: float = 0.15
    seed: int = 0
    dynamic_chunk: int = 3  # index of the recompute chunk (dynamic content mid-prompt)
    profile_noise: float = 0.05
    dtype: torch.dtype = torch.bfloat16


class RequestData:
    """Device tensors of one request (one layer)."""


class SyntheticWorkload:
    """Seeded C2-shaped inputs: Q, K ~ N(0,1)/sqrt(D), V ~ N(0,1), E ~ N(0, .02).

    Each request has ``chunks`` equal chunks, one recompute chunk and the
    rest reused; its paged blocks are a random permutation of a shared pool
    (with spare blocks for decode).
    """

    def __init__(self, cfg: WorkloadConfig, device: torch.device):
        self.cfg = cfg
        self.device = device
        g = torch.Generator().manual_seed(cfg.seed)
        n, hq, hkv, d, bs = cfg.seq, cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.block
        dt = cfg.dtype
        self.E = (torch.randn(d, cfg.npos, generator=g) * 0.02).to(device)
        blocks_per_req = (n + 1 + bs - 1) // bs + 1  # +1 block for decode tokens
        total_blocks = blocks_per_req * cfg.requests + 4
        self.cache = torch.zeros(total_blocks, hkv, bs, 2 * d, dtype=dt, device=device)
        pool = torch.randperm(total_blocks, generator=g)
        clen = n // cfg.chunks
        dyn = cfg.dynamic_chunk % cfg.chunks
        self.requests: list[RequestData] = []
        for b in range(cfg.requests):
            r = RequestData()
            r.block_table = pool[b * blocks_per_req:(b + 1) * blocks_per_req].to(device)
            tok = torch.arange(n + 1, device=device)
            r.slots_all = r.block_table[tok // bs] * bs + tok % bs
            r.slots = r.slots_all[:n].contiguous()
            chunk_of = torch.clamp(torch.arange(n) // clen, max=cfg.chunks - 1)
            r.key_chunk = chunk_of.to(torch.int32).to(device)
            reused = chunk_of != dyn
            mandatory = ~reused
            mandatory[n - 1] = True
            r.reused = reused.to(device)
            r.mandatory = mandatory.to(device)
            r.fixed = torch.nonzero(reused).flatten().to(device)
            r.cached_k = (torch.randn(n, hkv, d, generator=g) / math.sqrt(d)).to(dt).to(device)
            r.cached_v = torch.randn(n, hkv, d, generator=g).to(dt).to(device)
            # recomputed K at the calibration layer: profile K + N(0, noise)
            noise = cfg.profile_noise * torch.randn(n, hkv, d, generator=g)
            r.calib_k = (r.cached_k.float().cpu() + noise).to(dt).to(device)
            r.calib_k[r.mandatory] = r.cached_k[r.mandatory]
            # current-layer queries and fresh K/V for every token (rows sliced later)
            r.q_all = (torch.randn(n, hq, d, generator=g) / math.sqrt(d)).to(dt).to(device)
            r.fresh_k = (r.cached_k.float().cpu() + cfg.profile_noise *
                         torch.randn(n, hkv, d, generator=g)).to(dt).to(device)
            r.fresh_v = (r.cached_v.float().cpu() + cfg.profile_noise *
                         torch.randn(n, hkv, d, generator=g)).to(dt).to(device)
            # canonical carried counts per (head, token, chunk): the cached
            # layout's running count of an average gate (0.5 per token) from the
            # end of chunk c to the token; the token's own and later chunks carry
            pos = torch.arange(n, dtype=torch.float32)
            ends = torch.tensor([(c + 1) * clen - 1 for c in range(cfg.chunks)],
                                dtype=torch.float32)
            off = 0.5 * (pos[:, None] - ends[None, :])
            jitter = 1 + 0.05 * torch.randn(hq, n, cfg.chunks, generator=g)
            off = (off[None] * jitter).clamp_min(0)
            own_or_later = torch.arange(cfg.chunks)[None, :] >= chunk_of[:, None]
            off[:, own_or_later] = -1.0
            off[:, ~reused] = -1.0  # dynamic query rows use their actual counts
            r.offsets = off.to(device)
            r.decode_q = (torch.randn(1, hq, d, generator=g) / math.sqrt(d)).to(dt).to(device)
            r.decode_k = (torch.randn(1, hkv, d, generator=g) / math.sqrt(d)).to(dt).to(device)
            r.decode_v = torch.randn(1, hkv, d, generator=g).to(dt).to(device)
            self.requests.append(r)
        self.E_acc = self.E.float().contiguous()


def _i64(t: torch.Tensor) -> int:
    return t.data_ptr()


class ReuseStep:
    """All launches of one reuse-prefill layer for every request of a workload.

    ``batched_attention``: the CCPE attention of all requests runs as one
    launch (``cs_cope_attn_prefill_batch``, heaviest query tiles of every
    request first) once every request's WCA / SLIDE chain is done, instead of
    one launch per request on the request's stream (the default: the
    per-request launches overlap the other requests' WCA / SLIDE kernels).

    ``batched``: every stage runs as one launch for all requests on the
    caller's stream -- snapshot scatter (``cs_slide_scatter_batch``), WCA
    initialize, select, update and commit (``cs_wca_*_batch``) and the
    attention -- seven launches per step whatever the request count."""

    def __init__(self, work: SyntheticWorkload, batched_attention: bool = False,
                 batched: bool = False):
        self.work = work
        self.batched = batched
        self.batched_attention = batched_attention or batched
        cfg = work.cfg
        dev = work.device
        self.lib = N.load()
        self.status = torch.zeros(len(work.requests), dtype=torch.int32, device=dev)
        self.kv = N.paged_view(work.cache)
        n, hq, hkv, d = cfg.seq, cfg.q_heads, cfg.kv_heads, cfg.head_dim
        for b, r in enumerate(work.requests):
            r.dev = torch.empty(n, dtype=torch.float64, device=dev)
            r.alpha = torch.empty_like(r.dev)
            r.candidate = torch.zeros(n, dtype=torch.bool, device=dev)
            r.selected = torch.zeros_like(r.candidate)
            r.removed = torch.zeros_like(r.candidate)
            r.counts = torch.zeros(2, dtype=torch.int64, device=dev)
            r.counts2 = torch.zeros(2, dtype=torch.int64, device=dev)
            r.promoted = torch.empty(n, dtype=torch.int64, device=dev)
            r.removed_list = torch.empty(n, dtype=torch.int64, device=dev)
            r.status_ptr = self.status[b:b + 1].data_ptr()
        # one synchronised pass decides the budget and the active rows; the
        # timed launches recompute the same selection on the device
        self._initialize_all(stream=N.stream_of(dev))
        torch.cuda.synchronize(dev)
        for r in work.requests:
            reused, cand = r.counts.tolist()
            r.budget = min(math.ceil(cfg.fraction * reused), cand)
            self._select(r, N.stream_of(dev))
        torch.cuda.synchronize(dev)
        for r in work.requests:
            r.selected_prev = torch.nonzero(r.selected & ~r.mandatory).flatten()
            r.active = torch.nonzero(r.selected | r.mandatory).flatten()
            a = r.active.numel()
            r.a = a
            r.q = r.q_all[r.active].contiguous()
            r.fk = r.fresh_k[r.active].contiguous()
            r.fv = r.fresh_v[r.active].contiguous()
            r.active_slots = r.slots[r.active].contiguous()
            r.next_alpha = torch.empty(a, dtype=torch.float64, device=dev)
            r.used_alpha = torch.empty_like(r.next_alpha)
            r.cos = torch.empty_like(r.next_alpha)
            r.out = torch.empty(a, hq, d, dtype=cfg.dtype, device=dev)
            r.q_sel = torch.isin(r.active, r.selected_prev).to(torch.uint8)
            r.k_fix = r.reused.to(torch.uint8)
            r.co = r.offsets.index_select(1, r.active).contiguous()
            r.params = self._attn_params(r)
            # decode: query position n over n+1 keys (plain contextual)
            r.dec_slots = r.slots_all.contiguous()
            r.dec_out = torch.empty(1, hq, d, dtype=cfg.dtype, device=dev)
            r.dec_pos = torch.tensor([n], dtype=torch.int64, device=dev)
            r.dec_params = self._decode_params(r)
        # decode of the whole batch: one scatter of the new tokens, one
        # batched split-key decode (three launches for all requests)
        reqs = work.requests
        self.dec_params = (N.AttnParams * len(reqs))(*[r.dec_params for r in reqs])
        self.attn_params = (N.AttnParams * len(reqs))(*[r.params for r in reqs])
        size = self.lib.cs_cope_attn_decode_batch_workspace(self.dec_params, len(reqs))
        self.dec_ws = torch.empty(max(size, 1), dtype=torch.uint8, device=dev) if size else None
        self.dec_k = torch.cat([r.decode_k for r in reqs]).contiguous()
        self.dec_v = torch.cat([r.decode_v for r in reqs]).contiguous()
        self.dec_slots = torch.stack([r.slots_all[n] for r in reqs]).contiguous()
        self.gate_layer = True  # exercise the cosine gate in every timed step
        self._batch_items()
        # one stream per request: the launch chains touch disjoint slots of the
        # shared pool and their own WCA state, so they overlap on the device
        self.streams = [torch.cuda.Stream(device=dev) for _ in reqs]
        self._fork = torch.cuda.Event()
        self._joins = [torch.cuda.Event() for _ in reqs]

    def _batch_items(self) -> None:
        """The per-request arguments of the batched launches (all pointers
        stay valid for the step's lifetime)."""
        c, reqs = self.work.cfg, self.work.requests
        p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        self.scatter_items = (N.ScatterItem * len(reqs))(*[N.ScatterItem(
            p(r.slots), None, c.seq, p(r.cached_k), p(r.cached_v), r.cached_k.stride(0),
            r.cached_k.stride(1), r.status_ptr) for r in reqs])
        self.init_items = (N.InitializeItem * len(reqs))(*[N.InitializeItem(
            p(r.cached_k), r.cached_k.stride(0), r.cached_k.stride(1), p(r.calib_k),
            r.calib_k.stride(0), r.calib_k.stride(1), c.seq, p(r.reused), p(r.dev), p(r.alpha),
            p(r.candidate), p(r.selected), p(r.removed), p(r.counts), r.status_ptr)
            for r in reqs])
        self.select_items = (N.CommitItem * len(reqs))(*[N.CommitItem(
            None, 0, None, None, c.seq, r.budget, p(r.dev), p(r.alpha), p(r.candidate),
            p(r.selected), p(r.removed), None, p(r.promoted), p(r.counts2), r.status_ptr)
            for r in reqs])
        self.update_items = (N.UpdateItem * len(reqs))(*[N.UpdateItem(
            p(r.cached_k), p(r.cached_v), r.cached_k.stride(0), r.cached_k.stride(1), p(r.fk),
            p(r.fv), r.fk.stride(0), r.fk.stride(1), p(r.active), r.a, p(r.alpha),
            p(r.mandatory), None, None, p(r.next_alpha), p(r.used_alpha),
            p(r.cos) if self.gate_layer else None, p(r.active_slots), r.status_ptr)
            for r in reqs])
        self.commit_items = (N.CommitItem * len(reqs))(*[N.CommitItem(
            p(r.active), r.a, p(r.next_alpha), p(r.cos) if self.gate_layer else None, c.seq,
            r.budget, p(r.dev), p(r.alpha), p(r.candidate), p(r.selected), p(r.removed),
            p(r.removed_list), p(r.promoted), p(r.counts2), r.status_ptr) for r in reqs])

    # -------------------------------------------------------------- batched
    def scatter_all(self, stream) -> None:
        N.check(self.lib.cs_slide_scatter_batch(
            ctypes.byref(self.kv), self.scatter_items, len(self.scatter_items), stream),
            "cs_slide_scatter_batch")

    def initialize_all(self, stream) -> None:
        c = self.work.cfg
        N.check(self.lib.cs_wca_initialize_batch(
            self.init_items, len(self.init_items), c.kv_heads, c.head_dim, N.DTYPES[c.dtype],
            1e-8, 0, stream), "cs_wca_initialize_batch")

    def select_all(self, stream) -> None:
        N.check(self.lib.cs_wca_commit_batch(
            self.select_items, len(self.select_items), 0.12, 0, stream), "cs_wca_commit_batch")

    def update_all(self, stream) -> None:
        c = self.work.cfg
        N.check(self.lib.cs_wca_update_batch(
            self.update_items, len(self.update_items), c.kv_heads, c.head_dim,
            N.DTYPES[c.dtype], 0, 1e-8, 0, ctypes.byref(self.kv), stream),
            "cs_wca_update_batch")

    def commit_all(self, stream) -> None:
        N.check(self.lib.cs_wca_commit_batch(
            self.commit_items, len(self.commit_items), 0.12, 0, stream), "cs_wca_commit_batch")

    # -------------------------------------------------------------- pieces
    def _initialize_all(self, stream) -> None:
        for r in self.work.requests:
            self._initialize(r, stream)

    def _initialize(self, r, stream) -> None:
        cfg = self.work.cfg
        c, f = r.cached_k, r.calib_k
        N.check(self.lib.cs_wca_initialize(
            c.data_ptr(), c.stride(0), c.stride(1), f.data_ptr(), f.stride(0), f.stride(1),
            cfg.seq, cfg.kv_heads, cfg.head_dim, N.DTYPES[cfg.dtype], r.reused.data_ptr(), 1e-8,
            0, r.dev.data_ptr(), r.alpha.data_ptr(), r.candidate.data_ptr(),
            r.selected.data_ptr(), r.removed.data_ptr(), r.counts.data_ptr(), r.status_ptr,
            stream), "cs_wca_initialize")

    def _select(self, r, stream) -> None:
        N.check(self.lib.cs_wca_commit(
            None, 0, None, None, 0.12, 0, self.work.cfg.seq, r.budget, r.dev.data_ptr(),
            r.alpha.data_ptr(), r.candidate.data_ptr(), r.selected.data_ptr(),
            r.removed.data_ptr(), None, r.promoted.data_ptr(), r.counts2.data_ptr(),
            r.status_ptr, stream), "cs_wca_commit")

    def _attn_params(self, r) -> N.AttnParams:
        cfg = self.work.cfg
        p = N.AttnParams()
        p.q = r.q.data_ptr()
        p.q_stride_tok, p.q_stride_head = r.q.stride(0), r.q.stride(1)
        p.nq, p.hq, p.d = r.a, cfg.q_heads, cfg.head_dim
        p.qpos = r.active.data_ptr()
        p.paged = self.kv
        p.kv_slots = r.slots.data_ptr()
        p.nk, p.hkv, p.dv = cfg.seq, cfg.kv_heads, cfg.head_dim
        p.kpos = None
        p.E = self.work.E_acc.data_ptr()
        p.e_stride_d, p.e_stride_p = self.work.E_acc.stride()
        p.npos = cfg.npos
        p.scale = math.sqrt(cfg.head_dim)
        p.pos_mode = N.POS_CHUNK
        p.key_chunk = r.key_chunk.data_ptr()
        p.chunk_off = r.co.data_ptr()
        p.co_stride_h, p.co_stride_q = r.co.stride(0), r.co.stride(1)
        p.nchunks = cfg.chunks
        p.q_selected = r.q_sel.data_ptr()
        p.k_fixed = r.k_fix.data_ptr()
        p.atol = 1e-6
        p.out = r.out.data_ptr()
        p.o_stride_tok, p.o_stride_head = r.out.stride(0), r.out.stride(1)
        p.in_dtype = p.out_dtype = N.DTYPES[cfg.dtype]
        p.status = r.status_ptr
        return p

    def _decode_params(self, r) -> N.AttnParams:
        cfg = self.work.cfg
        p = N.AttnParams()
        p.q = r.decode_q.data_ptr()
        p.q_stride_tok, p.q_stride_head = r.decode_q.stride(0), r.decode_q.stride(1)
        p.nq, p.hq, p.d = 1, cfg.q_heads, cfg.head_dim
        p.qpos = r.dec_pos.data_ptr()
        p.paged = self.kv
        p.kv_slots = r.dec_slots.data_ptr()
        p.nk, p.hkv, p.dv = cfg.seq + 1, cfg.kv_heads, cfg.head_dim
        p.E = self.work.E_acc.data_ptr()
        p.e_stride_d, p.e_stride_p = self.work.E_acc.stride()
        p.npos = cfg.npos
        p.scale = math.sqrt(cfg.head_dim)
        p.out = r.dec_out.data_ptr()
        p.o_stride_tok, p.o_stride_head = r.dec_out.stride(0), r.dec_out.stride(1)
        p.in_dtype = p.out_dtype = N.DTYPES[cfg.dtype]
        p.status = r.status_ptr
        # decode() launches it right after the scatter of the newest records,
        # which writes no input the decode reads before waiting for it
        p.launch_flags = N.LAUNCH_OVERLAP_PREV
        return p

    # ------------------------------------------------------------- launches
    def baseline_write(self, r, stream) -> None:
        c = self.work.cfg
        N.check(self.lib.cs_slide_scatter(
            ctypes.byref(self.kv), r.slots.data_ptr(), None, c.seq, r.cached_k.data_ptr(),
            r.cached_v.data_ptr(), r.cached_k.stride(0), r.cached_k.stride(1), r.status_ptr,
            stream), "cs_slide_scatter")

    def wca_update(self, r, stream) -> None:
        c = self.work.cfg
        N.check(self.lib.cs_wca_update(
            r.cached_k.data_ptr(), r.cached_v.data_ptr(), r.cached_k.stride(0),
            r.cached_k.stride(1), r.fk.data_ptr(), r.fv.data_ptr(), r.fk.stride(0),
            r.fk.stride(1), r.active.data_ptr(), r.a, c.kv_heads, c.head_dim,
            N.DTYPES[c.dtype], r.alpha.data_ptr(), r.mandatory.data_ptr(), 0, 1e-8, 0, None,
            None, r.next_alpha.data_ptr(), r.used_alpha.data_ptr(),
            r.cos.data_ptr() if self.gate_layer else None, ctypes.byref(self.kv),
            r.active_slots.data_ptr(), r.status_ptr, stream), "cs_wca_update")

    def wca_commit(self, r, stream) -> None:
        c = self.work.cfg
        N.check(self.lib.cs_wca_commit(
            r.active.data_ptr(), r.a, r.next_alpha.data_ptr(),
            r.cos.data_ptr() if self.gate_layer else None, 0.12, 0, c.seq, r.budget,
            r.dev.data_ptr(), r.alpha.data_ptr(), r.candidate.data_ptr(),
            r.selected.data_ptr(), r.removed.data_ptr(), r.removed_list.data_ptr(),
            r.promoted.data_ptr(), r.counts2.data_ptr(), r.status_ptr, stream),
            "cs_wca_commit")

    def attention(self, r, stream) -> None:
        rc = self.lib.cs_cope_attn_prefill(ctypes.byref(r.params), stream)
        if rc == N.CS_ERR_UNSUPPORTED:
            rc = self.lib.cs_cope_attn(ctypes.byref(r.params), stream)
        N.check(rc, "attention")

    def attention_all(self, stream) -> None:
        """The attention of every request in one launch."""
        reqs = self.work.requests
        rc = self.lib.cs_cope_attn_prefill_batch(self.attn_params, len(reqs), stream)
        if rc == N.CS_ERR_UNSUPPORTED:
            for r in reqs:
                self.attention(r, stream)
            return
        N.check(rc, "cs_cope_attn_prefill_batch")

    def run(self, stream: int | None = None, before=None, after=None,
            batched: bool | None = None) -> list[torch.Tensor]:
        """One reuse-prefill layer for every request; returns the outputs.

        Each request's launches go to its own stream, which first waits for
        the caller's stream (``stream`` handle, default the current one); the
        caller's stream then waits for every request, so work queued on it
        afterwards sees all outputs.  ``before(request, stream)`` and
        ``after(request, stream)`` run with that request's stream current
        around its launches (host <-> device staging of its tensors).
        ``batched`` overrides the step's schedule for this call (the batched
        launches, or the per-request streams whose staging copies overlap
        the other requests' kernels)."""
        dev = self.work.device
        main = (torch.cuda.current_stream(dev) if stream is None
                else torch.cuda.ExternalStream(stream, device=dev))
        if self.batched if batched is None else batched:
            s = main.cuda_stream
            if before is not None:
                for r in self.work.requests:
                    before(r, main)
            self.scatter_all(s)
            self.initialize_all(s)
            self.select_all(s)
            self.update_all(s)
            self.commit_all(s)
            self.attention_all(s)
            if after is not None:
                for r in self.work.requests:
                    after(r, main)
            return [r.out for r in self.work.requests]
        self._fork.record(main)
        batched = self.batched_attention and batched is not False
        for r, rs, done in zip(self.work.requests, self.streams, self._joins):
            rs.wait_event(self._fork)
            s = rs.cuda_stream
            if before is not None:
                with torch.cuda.stream(rs):
                    before(r, rs)
            self.baseline_write(r, s)
            self._initialize(r, s)
            self._select_async(r, s)
            self.wca_update(r, s)
            self.wca_commit(r, s)
            if not batched:
                self.attention(r, s)
                if after is not None:
                    with torch.cuda.stream(rs):
                        after(r, rs)
            done.record(rs)
        for done in self._joins:
            main.wait_event(done)
        if batched:
            self.attention_all(main.cuda_stream)
            if after is not None:
                with torch.cuda.stream(main):
                    for r in self.work.requests:
                        after(r, main)
        return [r.out for r in self.work.requests]

    def _select_async(self, r, s) -> None:
        # cs_wca_initialize restarted selected/removed from zero (fresh state)
        self._select(r, s)

    def decode(self, stream: int | None = None) -> list[torch.Tensor]:
        """One decode token per request: write the new K/V rows of all
        requests (one scatter into the shared pool), then attend over n+1 keys
        for every request in one batched split-key decode."""
        s = N.stream_of(self.work.device) if stream is None else stream
        reqs = self.work.requests
        N.check(self.lib.cs_slide_scatter(
            ctypes.byref(self.kv), self.dec_slots.data_ptr(), None, len(reqs),
            self.dec_k.data_ptr(), self.dec_v.data_ptr(), self.dec_k.stride(0),
            self.dec_k.stride(1), reqs[0].status_ptr, s), "cs_slide_scatter")
        rc = N.CS_ERR_UNSUPPORTED
        if self.dec_ws is not None:
            rc = self.lib.cs_cope_attn_decode_batch(self.dec_params, len(reqs),
                                                    self.dec_ws.data_ptr(), s)
        if rc == N.CS_ERR_UNSUPPORTED:
            for r in reqs:
                N.check(self.lib.cs_cope_attn(ctypes.byref(r.dec_params), s), "decode")
        else:
            N.check(rc, "cs_cope_attn_decode_batch")
        return [r.dec_out for r in reqs]

    def check_status(self) -> None:
        """Raise if any launch of any request reported a status bit."""
        acc = 0
        for word in self.status.cpu().tolist():
            acc |= int(word)
        if acc:
            raise RuntimeError(f"device status bits set: {acc:#x}")


def dense_inputs(work: SyntheticWorkload, b: int, step: ReuseStep):
    """Dense q, fused K/V and query positions of request b after a step
    (gathered back from the paged cache) -- for oracle checks."""
    r = work.requests[b]
    c = work.cfg
    k = torch.empty(c.seq, c.kv_heads, c.head_dim, dtype=c.dtype, device=work.device)
    v = torch.empty_like(k)
    st = torch.zeros(1, dtype=torch.int32, device=work.device)
    N.check(step.lib.cs_slide_gather(
        ctypes.byref(step.kv), r.slots.data_ptr(), c.seq, k.data_ptr(), v.data_ptr(),
        k.stride(0), k.stride(1), st.data_ptr(), N.stream_of(work.device)), "gather")
    torch.cuda.synchronize(work.device)
    return r.q, k, v, r.active
