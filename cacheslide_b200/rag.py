"""A retrieval-augmented batch with shared document chunks (the C3 layout).

A pool of ``pool_chunks`` document chunks (512 tokens each) is resident once
in the paged pool; each request retrieves ``chunks_per_request`` distinct
chunks drawn by a Zipf(1.1) popularity over the pool, in random order, and
appends a 64-token question.  The requests' block tables share the chunks'
physical blocks, so a popular chunk's KV is stored once however many
requests read it.  The turn (``chat._TurnStep``) then runs per request:
WCA over the prompt (the question's rows mandatory, 15 % of the chunk rows
selected), copy-on-write relocation of the selected chunk rows into the
request's private slots (the shared blocks are never written), the blend,
the attention of the active rows through the request's slot table, and 32
decode steps.  (The reference's RAG evaluation uses HotpotQA, absent here;
only its shape is used.)
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch

from .chat import _Session, _TurnStep


@dataclass(frozen=True)
class RagConfig:
    requests: int = 64
    pool_chunks: int = 40
    chunks_per_request: int = 10
    chunk_tokens: int = 512
    question_tokens: int = 64
    zipf: float = 1.1
    q_heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    npos: int = 64
    block: int = 16
    fraction: float = 0.15
    decode_tokens: int = 32
    seed: int = 0
    dtype: torch.dtype = torch.bfloat16


class RagStep(_TurnStep):
    """The reuse prefill and answer decode of a RAG batch (see the module)."""

    def __init__(self, cfg: RagConfig, device: torch.device):
        hkv, d, bs = cfg.kv_heads, cfg.head_dim, cfg.block
        dt = cfg.dtype
        if cfg.chunk_tokens % bs:
            raise ValueError("chunks must fill whole blocks")
        lay = torch.Generator().manual_seed(cfg.seed)
        g = torch.Generator(device=device).manual_seed(cfg.seed + 1)
        cb = cfg.chunk_tokens // bs  # blocks a chunk
        tail = cfg.question_tokens + cfg.decode_tokens
        qb = (tail + bs - 1) // bs
        n = cfg.chunks_per_request * cfg.chunk_tokens + cfg.question_tokens
        reused_rows = cfg.chunks_per_request * cfg.chunk_tokens
        pb = (math.ceil(cfg.fraction * reused_rows) + bs) // bs + 1
        total_blocks = cfg.pool_chunks * cb + cfg.requests * (qb + pb)
        perm = torch.randperm(total_blocks, generator=lay).to(device)
        chunk_blocks = perm[: cfg.pool_chunks * cb].view(cfg.pool_chunks, cb)
        rest = perm[cfg.pool_chunks * cb:]
        cache = torch.zeros(total_blocks, hkv, bs, 2 * d, dtype=dt, device=device)
        # the pool's chunk content, once
        ck = (torch.randn(cfg.pool_chunks, cfg.chunk_tokens, hkv, d, generator=g, device=device)
              / math.sqrt(d)).to(dt)
        cv = torch.randn(cfg.pool_chunks, cfg.chunk_tokens, hkv, d, generator=g,
                         device=device).to(dt)
        weights = 1.0 / torch.arange(1, cfg.pool_chunks + 1, dtype=torch.float64) ** cfg.zipf
        self.chunk_reads = torch.zeros(cfg.pool_chunks, dtype=torch.int64)
        sessions = []
        tok_in = torch.arange(cfg.chunk_tokens, device=device)
        for b in range(cfg.requests):
            picks = torch.multinomial(weights, cfg.chunks_per_request, replacement=False,
                                      generator=lay)
            picks = picks[torch.randperm(picks.numel(), generator=lay)]
            self.chunk_reads[picks] += 1
            s = _Session()
            s.n, s.new = n, cfg.question_tokens
            own = rest[b * (qb + pb):(b + 1) * (qb + pb)]
            qblocks, s.private_blocks = own[:qb], own[qb:]
            parts = [chunk_blocks[c][tok_in // bs] * bs + tok_in % bs for c in picks.tolist()]
            t = torch.arange(tail, device=device)
            parts.append(qblocks[t // bs] * bs + t % bs)
            s.slots_all = torch.cat(parts).contiguous()
            s.reused = torch.zeros(n, dtype=torch.bool, device=device)
            s.reused[:reused_rows] = True
            qk = (torch.randn(cfg.question_tokens, hkv, d, generator=g, device=device)
                  / math.sqrt(d)).to(dt)
            qv = torch.randn(cfg.question_tokens, hkv, d, generator=g, device=device).to(dt)
            s.cached_k = torch.cat([ck[picks.to(device)].reshape(-1, hkv, d), qk]).contiguous()
            s.cached_v = torch.cat([cv[picks.to(device)].reshape(-1, hkv, d), qv]).contiguous()
            s.picks = picks
            sessions.append(s)
        super().__init__(cfg, device, cache, sessions, g)

    def shared_fraction(self) -> float:
        """Chunk reads served by a block another request also reads."""
        reads = self.chunk_reads
        return float((reads[reads > 1]).sum()) / float(reads.sum())
