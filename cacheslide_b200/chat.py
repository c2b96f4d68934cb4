"""One turn of the multi-session chat slice (the C4 layout).

S sessions, each at turn t of a conversation whose turns add 256-1024 user
tokens plus 128 decoded tokens.  A session's history (all earlier turns) is
resident in its paged blocks; the turn is one reuse-prefill layer and then
the decode of its answer:

1. WCA over the prompt (history + the new message): deviation of the cached
   K against the calibration K, the selection of the history rows to
   recompute (15 %), the new message's rows mandatory
   (``cs_wca_initialize_batch``, ``cs_wca_commit_batch``);
2. SLIDE relocation: the selected history rows' records are copied out of
   their canonical slots into private slots of the session (the reference
   promotes selected tokens out of the shared snapshot before updating them,
   paged.py:279-328), ``cs_slide_relocate`` per session;
3. the blend of the recomputed rows into their slots -- private slots for the
   selected history rows, canonical ones for the new message
   (``cs_wca_update_batch``), and the commit;
4. CCPE attention of the active rows over the prompt through the turn's slot
   table (selected history -> private slots), all sessions in one launch;
5. 128 decode steps for all sessions: the new token's K/V scattered into its
   canonical slot, then the batched split-key decode over the grown context.

Every session has its own length; the batched launches take ragged items.
A first pass at construction fixes the selection (as ``reuse.ReuseStep``
does), so the relocation lists and the attention arguments are built once.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass

import torch

from . import _native as N


@dataclass(frozen=True)
class ChatConfig:
    sessions: int = 32
    turn: int = 8
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    min_tokens: int = 256
    max_tokens: int = 1024
    decode_tokens: int = 128
    npos: int = 64
    block: int = 16
    fraction: float = 0.15
    seed: int = 0
    dtype: torch.dtype = torch.bfloat16


class _Session:
    """Device tensors of one session."""


class _TurnStep:
    """The launches of a reuse turn over sessions whose reused rows are
    resident in paged slots (``slots_all[:n]``, possibly shared between
    sessions with identical records) and whose dynamic rows and decoded
    tokens have slots of their own: WCA, copy-on-write relocation of the
    selected reused rows into the session's ``private_blocks``, blend,
    attention, decode (see the module)."""

    def __init__(self, cfg, device: torch.device, cache: torch.Tensor, sessions: list,
                 g: torch.Generator):
        self.cfg, self.device = cfg, device
        self.lib = N.load()
        hq, hkv, d, bs = cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.block
        dt = cfg.dtype

        def randn(*shape, scale=1.0):
            return (torch.randn(*shape, generator=g, device=device) * scale).to(dt)

        self.cache = cache
        self.kv = N.paged_view(self.cache)
        self.E = (torch.randn(d, cfg.npos, generator=g, device=device) * 0.02).contiguous()
        self.status = torch.zeros(len(sessions), dtype=torch.int32, device=device)
        self.sessions = sessions
        for b, s in enumerate(sessions):
            n = s.n
            s.hist = int(s.reused.sum())
            s.canon = s.slots_all[:n].contiguous()
            s.mandatory = ~s.reused
            s.calib_k = (s.cached_k.float() + 0.05 * torch.randn(
                n, hkv, d, generator=g, device=device)).to(dt)
            s.calib_k[s.mandatory] = s.cached_k[s.mandatory]
            s.fresh_k = (s.cached_k.float() + 0.05 * torch.randn(
                n, hkv, d, generator=g, device=device)).to(dt)
            s.fresh_v = (s.cached_v.float() + 0.05 * torch.randn(
                n, hkv, d, generator=g, device=device)).to(dt)
            s.dec_q = randn(cfg.decode_tokens, hq, d, scale=1 / math.sqrt(d))
            s.dec_k = randn(cfg.decode_tokens, hkv, d, scale=1 / math.sqrt(d))
            s.dec_v = randn(cfg.decode_tokens, hkv, d)
            s.dec_pos = torch.arange(n, n + cfg.decode_tokens, device=device)
            s.status_ptr = self.status[b:b + 1].data_ptr()
            for name in ("dev", "alpha"):
                setattr(s, name, torch.empty(n, dtype=torch.float64, device=device))
            for name in ("candidate", "selected", "removed"):
                setattr(s, name, torch.zeros(n, dtype=torch.bool, device=device))
            s.counts = torch.zeros(2, dtype=torch.int64, device=device)
            s.counts2 = torch.zeros(2, dtype=torch.int64, device=device)
            s.promoted = torch.empty(n, dtype=torch.int64, device=device)
            s.removed_list = torch.empty(n, dtype=torch.int64, device=device)
        # the resident history: every prompt record in its canonical slot
        for s in self.sessions:
            N.check(self.lib.cs_slide_scatter(
                ctypes.byref(self.kv), s.canon.data_ptr(), None, s.n, s.cached_k.data_ptr(),
                s.cached_v.data_ptr(), s.cached_k.stride(0), s.cached_k.stride(1),
                s.status_ptr, N.stream_of(device)), "cs_slide_scatter")
        # first pass: the selection, hence the relocation lists and slot tables
        self._items()
        st = N.stream_of(device)
        self.initialize_all(st)
        torch.cuda.synchronize(device)
        for s in self.sessions:
            reused, cand = s.counts.tolist()
            s.budget = min(math.ceil(cfg.fraction * reused), cand)
        self._select_items()
        self.select_all(st)
        torch.cuda.synchronize(device)
        for s in self.sessions:
            sel = torch.nonzero(s.selected & ~s.mandatory).flatten()
            s.active = torch.nonzero(s.selected | s.mandatory).flatten()
            s.a = s.active.numel()
            if sel.numel() > s.private_blocks.numel() * bs:
                raise ValueError("private blocks too small for the selection")
            ptok = torch.arange(sel.numel(), device=device)
            s.reloc_src = s.canon[sel].contiguous()
            s.reloc_dst = (s.private_blocks[ptok // bs] * bs + ptok % bs).contiguous()
            s.table = s.canon.clone()  # the turn's slot table: selected -> private
            s.table[sel] = s.reloc_dst
            tab_all = s.slots_all.clone()
            tab_all[:s.n] = s.table
            s.dec_table = tab_all
            s.active_slots = s.table[s.active].contiguous()
            s.q = randn(s.a, hq, d, scale=1 / math.sqrt(d))
            s.fk = s.fresh_k[s.active].contiguous()
            s.fv = s.fresh_v[s.active].contiguous()
            s.next_alpha = torch.empty(s.a, dtype=torch.float64, device=device)
            s.used_alpha = torch.empty_like(s.next_alpha)
            s.cos = torch.empty_like(s.next_alpha)
            s.out = torch.empty(s.a, hq, d, dtype=dt, device=device)
            s.selected_prev = sel
            s.q_sel = torch.isin(s.active, sel).to(torch.uint8)
            s.k_fix = s.reused.to(torch.uint8)
            s.params = self._attn_params(s)
            s.dec_out = torch.empty(cfg.decode_tokens, hq, d, dtype=dt, device=device)
        self._update_items()
        self.attn_params = (N.AttnParams * len(self.sessions))(*[s.params for s in self.sessions])
        # decode: one params array per step (the context grows by one key)
        self.dec_params = []
        for t in range(cfg.decode_tokens):
            arr = (N.AttnParams * len(self.sessions))(*[self._decode_params(s, t)
                                                  for s in self.sessions])
            self.dec_params.append(arr)
        size = max(self.lib.cs_cope_attn_decode_batch_workspace(p, len(self.sessions))
                   for p in (self.dec_params[0], self.dec_params[-1]))
        self.dec_ws = torch.empty(max(size, 1), dtype=torch.uint8, device=device)
        self.dec_rows = torch.stack([s.slots_all[s.n:] for s in self.sessions], 1).contiguous()
        self.dec_k = torch.stack([s.dec_k for s in self.sessions], 1).contiguous()
        self.dec_v = torch.stack([s.dec_v for s in self.sessions], 1).contiguous()
        torch.cuda.synchronize(device)

    # ------------------------------------------------------------ arguments
    def _items(self) -> None:
        c = self.cfg
        p = lambda t: None if t is None else t.data_ptr()  # noqa: E731
        self.init_items = (N.InitializeItem * len(self.sessions))(*[N.InitializeItem(
            p(s.cached_k), s.cached_k.stride(0), s.cached_k.stride(1), p(s.calib_k),
            s.calib_k.stride(0), s.calib_k.stride(1), s.n, p(s.reused), p(s.dev), p(s.alpha),
            p(s.candidate), p(s.selected), p(s.removed), p(s.counts), s.status_ptr)
            for s in self.sessions])

    def _select_items(self) -> None:
        p = lambda t: t.data_ptr()  # noqa: E731
        self.select_items = (N.CommitItem * len(self.sessions))(*[N.CommitItem(
            None, 0, None, None, s.n, s.budget, p(s.dev), p(s.alpha), p(s.candidate),
            p(s.selected), p(s.removed), None, p(s.promoted), p(s.counts2), s.status_ptr)
            for s in self.sessions])

    def _update_items(self) -> None:
        p = lambda t: t.data_ptr()  # noqa: E731
        self.update_items = (N.UpdateItem * len(self.sessions))(*[N.UpdateItem(
            p(s.cached_k), p(s.cached_v), s.cached_k.stride(0), s.cached_k.stride(1), p(s.fk),
            p(s.fv), s.fk.stride(0), s.fk.stride(1), p(s.active), s.a, p(s.alpha),
            p(s.mandatory), None, None, p(s.next_alpha), p(s.used_alpha), p(s.cos),
            p(s.active_slots), s.status_ptr) for s in self.sessions])
        self.commit_items = (N.CommitItem * len(self.sessions))(*[N.CommitItem(
            p(s.active), s.a, p(s.next_alpha), p(s.cos), s.n, s.budget, p(s.dev), p(s.alpha),
            p(s.candidate), p(s.selected), p(s.removed), p(s.removed_list), p(s.promoted),
            p(s.counts2), s.status_ptr) for s in self.sessions])

    def _attn_params(self, s) -> N.AttnParams:
        c = self.cfg
        p = N.AttnParams()
        p.q = s.q.data_ptr()
        p.q_stride_tok, p.q_stride_head = s.q.stride(0), s.q.stride(1)
        p.nq, p.hq, p.d = s.a, c.q_heads, c.head_dim
        p.qpos = s.active.data_ptr()
        p.paged = self.kv
        p.kv_slots = s.table.data_ptr()
        p.nk, p.hkv, p.dv = s.n, c.kv_heads, c.head_dim
        p.E = self.E.data_ptr()
        p.e_stride_d, p.e_stride_p = self.E.stride()
        p.npos = c.npos
        p.scale = math.sqrt(c.head_dim)
        p.q_selected = s.q_sel.data_ptr()
        p.k_fixed = s.k_fix.data_ptr()
        p.atol = 1e-6
        p.out = s.out.data_ptr()
        p.o_stride_tok, p.o_stride_head = s.out.stride(0), s.out.stride(1)
        p.in_dtype = p.out_dtype = N.DTYPES[c.dtype]
        p.status = s.status_ptr
        return p

    def _decode_params(self, s, t: int) -> N.AttnParams:
        c = self.cfg
        p = N.AttnParams()
        q = s.dec_q[t:t + 1]
        p.q = q.data_ptr()
        p.q_stride_tok, p.q_stride_head = q.stride(0), q.stride(1)
        p.nq, p.hq, p.d = 1, c.q_heads, c.head_dim
        p.qpos = s.dec_pos[t:t + 1].data_ptr()
        p.paged = self.kv
        p.kv_slots = s.dec_table.data_ptr()
        p.nk, p.hkv, p.dv = s.n + t + 1, c.kv_heads, c.head_dim
        p.E = self.E.data_ptr()
        p.e_stride_d, p.e_stride_p = self.E.stride()
        p.npos = c.npos
        p.scale = math.sqrt(c.head_dim)
        out = s.dec_out[t:t + 1]
        p.out = out.data_ptr()
        p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
        p.in_dtype = p.out_dtype = N.DTYPES[c.dtype]
        p.status = s.status_ptr
        p.launch_flags = N.LAUNCH_OVERLAP_PREV  # after this library's scatter only
        return p

    # ------------------------------------------------------------- launches
    def initialize_all(self, stream) -> None:
        c = self.cfg
        N.check(self.lib.cs_wca_initialize_batch(
            self.init_items, len(self.sessions), c.kv_heads, c.head_dim, N.DTYPES[c.dtype], 1e-8, 0,
            stream), "cs_wca_initialize_batch")

    def select_all(self, stream) -> None:
        N.check(self.lib.cs_wca_commit_batch(self.select_items, len(self.sessions), 0.12, 0,
                                             stream), "cs_wca_commit_batch")

    def relocate_all(self, stream) -> None:
        for s in self.sessions:
            if s.reloc_src.numel():
                N.check(self.lib.cs_slide_relocate(
                    ctypes.byref(self.kv), s.reloc_src.data_ptr(), s.reloc_dst.data_ptr(),
                    s.reloc_src.numel(), s.status_ptr, stream), "cs_slide_relocate")

    def update_all(self, stream) -> None:
        c = self.cfg
        N.check(self.lib.cs_wca_update_batch(
            self.update_items, len(self.sessions), c.kv_heads, c.head_dim, N.DTYPES[c.dtype], 0, 1e-8,
            0, ctypes.byref(self.kv), stream), "cs_wca_update_batch")
        N.check(self.lib.cs_wca_commit_batch(self.commit_items, len(self.sessions), 0.12, 0, stream),
                "cs_wca_commit_batch")

    def attention_all(self, stream) -> None:
        N.check(self.lib.cs_cope_attn_prefill_batch(self.attn_params, len(self.sessions),
                                                    stream), "cs_cope_attn_prefill_batch")

    def prefill(self, stream) -> None:
        """Steps 1-4 of the module docstring."""
        self.initialize_all(stream)
        self.select_all(stream)
        self.relocate_all(stream)
        self.update_all(stream)
        self.attention_all(stream)

    def decode(self, stream, steps: int | None = None) -> None:
        """The answer's decode steps for all sessions."""
        c = self.cfg
        rows = self.dec_rows
        for t in range(c.decode_tokens if steps is None else steps):
            N.check(self.lib.cs_slide_scatter(
                ctypes.byref(self.kv), rows[t].data_ptr(), None, len(self.sessions),
                self.dec_k[t].data_ptr(), self.dec_v[t].data_ptr(), self.dec_k.stride(1),
                self.dec_k.stride(2), self.sessions[0].status_ptr, stream), "cs_slide_scatter")
            N.check(self.lib.cs_cope_attn_decode_batch(
                self.dec_params[t], len(self.sessions), self.dec_ws.data_ptr(), stream),
                "cs_cope_attn_decode_batch")

    def check_status(self) -> None:
        acc = 0
        for word in self.status.cpu().tolist():
            acc |= int(word)
        if acc:
            raise RuntimeError(f"device status bits set: {acc:#x}")

    def prompt_tokens(self) -> int:
        return sum(s.n for s in self.sessions)

    def new_tokens(self) -> int:
        return sum(s.new for s in self.sessions)


class ChatTurnStep(_TurnStep):
    """One chat turn for every session (see the module)."""

    def __init__(self, cfg: ChatConfig, device: torch.device):
        hq, hkv, d, bs = cfg.q_heads, cfg.kv_heads, cfg.head_dim, cfg.block
        dt = cfg.dtype
        lay = torch.Generator().manual_seed(cfg.seed)
        g = torch.Generator(device=device).manual_seed(cfg.seed + 1)

        def randn(*shape, scale=1.0):
            return (torch.randn(*shape, generator=g, device=device) * scale).to(dt)

        # session layouts: turn lengths, history, blocks (canonical + private)
        specs = []
        total_blocks = 0
        for _ in range(cfg.sessions):
            lens = torch.randint(cfg.min_tokens, cfg.max_tokens + 1, (cfg.turn,),
                                 generator=lay).tolist()
            turns = [x + cfg.decode_tokens for x in lens[:-1]] + [lens[-1]]
            n = sum(turns)
            hist = n - turns[-1]
            canon_blocks = (n + cfg.decode_tokens + bs - 1) // bs
            priv_blocks = (math.ceil(cfg.fraction * hist) + bs) // bs + 1
            specs.append((turns, n, hist, canon_blocks, priv_blocks))
            total_blocks += canon_blocks + priv_blocks
        pool = torch.randperm(total_blocks, generator=lay).to(device)
        cache = torch.zeros(total_blocks, hkv, bs, 2 * d, dtype=dt, device=device)
        sessions = []
        cursor = 0
        for turns, n, hist, cb, pb in specs:
            s = _Session()
            s.n, s.new = n, turns[-1]
            blocks = pool[cursor:cursor + cb]
            s.private_blocks = pool[cursor + cb:cursor + cb + pb]
            cursor += cb + pb
            tok = torch.arange(n + cfg.decode_tokens, device=device)
            s.slots_all = (blocks[tok // bs] * bs + tok % bs).contiguous()
            s.reused = (tok[:n] < hist).contiguous()
            s.cached_k = randn(n, hkv, d, scale=1 / math.sqrt(d))
            s.cached_v = randn(n, hkv, d)
            sessions.append(s)
        super().__init__(cfg, device, cache, sessions, g)
