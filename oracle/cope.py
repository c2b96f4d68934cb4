"""numpy restatement of CoPE / CCPE attention (TEST INFRASTRUCTURE ONLY).

Follows the reference ``src/cacheslide_vllm/position.py`` and
``src/cacheslide_vllm/attention.py``; each function names the lines it restates.
Arrays use the reference layouts: query ``[Nq, Hq, D]``, key/value
``[Nk, Hkv, D]``, positions/logits ``[H, Nq, Nk]``, learned table ``E [D, npos]``.
bf16/fp16 inputs are passed as their exact float32 upcast; float64 inputs keep
float64 accumulation, as the reference does (position.py:153-154).
"""

from __future__ import annotations

import math

import numpy as np

NONNEGATIVE = "causal contextual positions must be nonnegative"
AVAILABLE = "causal contextual count exceeds available gates"
NONINCREASING = "causal contextual path must be nonincreasing"
ONE_GATE = "causal contextual path exceeds one gate per token"


def acc_dtype(dtype) -> type:
    """position.py:153-154 -- float64 stays float64, everything else float32."""
    return np.float64 if np.dtype(dtype) == np.float64 else np.float32


def qk_logits(q: np.ndarray, k: np.ndarray) -> np.ndarray:
    """position.py:157-164 -- GQA logits ``[Hq, Nq, Nk]`` scaled by 1/sqrt(D).

    Query head h uses KV head h // group (``repeat_interleave``); the grouped
    matmul computes exactly that without materialising repeated keys.
    """
    a = acc_dtype(q.dtype)
    nq, hq, d = q.shape
    nk, hkv, _ = k.shape
    group = hq // hkv
    qg = q.astype(a).transpose(1, 0, 2).reshape(hkv, group * nq, d)
    kg = k.astype(a).transpose(1, 2, 0)  # [Hkv, D, Nk]
    logits = np.matmul(qg, kg).reshape(hq, nq, nk)
    return (logits / a(math.sqrt(d))).astype(a)


def causal_mask(qpos: np.ndarray, kpos: np.ndarray) -> np.ndarray:
    """position.py:180 -- key coordinate <= query coordinate, ``[Nq, Nk]``."""
    return kpos[None, :] <= qpos[:, None]


def sigmoid(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (1 / (1 + np.exp(-x))).astype(x.dtype)


def reverse_cumsum(gates: np.ndarray) -> np.ndarray:
    """``flip(-1).cumsum(-1).flip(-1)``; torch's CPU cumsum accumulates float32
    in float64 and rounds each prefix, which this reproduces."""
    acc = np.cumsum(gates[..., ::-1].astype(np.float64), axis=-1)[..., ::-1]
    return acc.astype(gates.dtype)


def contextual_positions(logits, allowed, npos: int) -> np.ndarray:
    """position.py:295-307 -- masked gates, reverse cumsum over keys, clamp."""
    gates = np.where(allowed, sigmoid(logits), logits.dtype.type(0))
    return np.clip(reverse_cumsum(gates), 0, npos - 1).astype(logits.dtype)


def chunk_reset_positions(
    logits, allowed, key_chunk, offsets, q_chunk, npos: int
) -> np.ndarray:
    """Compressed CCPE positions: the reverse gate sum restarts at every chunk
    boundary from a carried per-(head, query, chunk) offset.

    ``offsets[h, i, c] >= 0`` replaces the running count entering chunk ``c``
    (only for chunks older than the query's own chunk ``q_chunk[i]``); a
    negative offset carries the actual running count across the boundary, so
    all-negative offsets reproduce plain CoPE (position.py:295-307).
    """
    gates = np.where(allowed, sigmoid(logits), logits.dtype.type(0))
    out = np.zeros_like(gates)
    carry = np.zeros(gates.shape[:2], dtype=gates.dtype)
    nchunks = int(key_chunk.max()) + 1 if key_chunk.size else 0
    for c in range(nchunks - 1, -1, -1):
        cols = np.nonzero(key_chunk == c)[0]
        if cols.size == 0:
            continue
        local = reverse_cumsum(gates[..., cols])
        off = offsets[:, :, c]
        reset = (off >= 0) & (c < q_chunk[None, :])
        base = np.where(reset, off, carry).astype(gates.dtype)
        out[..., cols] = local + base[..., None]
        carry = out[..., cols[0]]
    return np.clip(out, 0, npos - 1).astype(gates.dtype)


def query_chunk_ids(qpos, kpos, key_chunk) -> np.ndarray:
    """Chunk of each query = chunk of its newest causal key (-1 if none)."""
    n = np.searchsorted(kpos, qpos, side="right")
    return np.where(n > 0, key_chunk[np.maximum(n - 1, 0)], -1)


def positional_bias(q, E, positions) -> np.ndarray:
    """position.py:309-344 -- ``q.E`` table, floor / floor+1 interpolation."""
    a = acc_dtype(q.dtype)
    npos = E.shape[1]
    table = np.einsum("qhd,dp->hqp", q.astype(a), E.astype(a)).astype(a)
    positions = positions.astype(a, copy=False)
    floor = np.floor(positions)
    lower = floor.astype(np.int32)
    upper = np.minimum(lower + 1, npos - 1)
    frac = positions - floor
    lo = np.take_along_axis(table, lower, axis=-1)
    hi = np.take_along_axis(table, upper, axis=-1)
    hi -= lo
    hi *= frac
    hi += lo
    return hi


def _head_mask(mask, heads, nq, nk):
    if mask is None:
        return None
    mask = np.asarray(mask, dtype=bool)
    if mask.ndim == 2:
        mask = mask[None]
    return np.broadcast_to(mask, (heads, nq, nk))


def cope_attention(
    q,
    k,
    v,
    E,
    qpos,
    kpos=None,
    *,
    gate_mask=None,
    vis_mask=None,
    positions_fn=None,
    visibility_fn=None,
    fixed_positions=None,
    chunk_reset=None,
    chunk: int = 128,
    return_positions: bool = False,
):
    """position.py:404-560 -- gates, position transform, bias, visibility,
    masked softmax (all-masked rows give zero), PV.

    ``chunk_reset=(key_chunk, offsets)`` replaces the contextual positions by
    ``chunk_reset_positions`` before any transform.  Returns the output in the
    accumulation dtype (the caller casts to the value dtype).
    """
    a = acc_dtype(q.dtype)
    nq, hq, _ = q.shape
    nk = k.shape[0]
    npos = E.shape[1]
    qpos = np.asarray(qpos, dtype=np.int64)
    kpos = np.arange(nk, dtype=np.int64) if kpos is None else np.asarray(kpos)
    gm = _head_mask(gate_mask, hq, nq, nk)
    vm = _head_mask(vis_mask, hq, nq, nk)
    hkv = v.shape[1]
    group = hq // hkv
    values = v.astype(a).transpose(1, 0, 2)  # [Hkv, Nk, Dv]; head h reads h // group
    outs, traces = [], []
    for start in range(0, nq, chunk):
        end = min(start + chunk, nq)
        qc, qp = q[start:end], qpos[start:end]
        allowed = np.broadcast_to(causal_mask(qp, kpos)[None], (hq, end - start, nk))
        if gm is not None:
            allowed = allowed & gm[:, start:end]
        logits = qk_logits(qc, k)
        if fixed_positions is not None:
            positions = np.asarray(fixed_positions, dtype=a)[:, start:end]
        elif chunk_reset is not None:
            key_chunk, offsets = chunk_reset
            qch = query_chunk_ids(qp, kpos, key_chunk)
            positions = chunk_reset_positions(
                logits, allowed, key_chunk, offsets[:, start:end], qch, npos
            )
        else:
            positions = contextual_positions(logits, allowed, npos)
        if positions_fn is not None:
            positions = np.asarray(positions_fn(positions, qp, kpos), dtype=a)
        scores = logits + positional_bias(qc, E, positions)
        visible = allowed
        if vm is not None:
            visible = visible & vm[:, start:end]
        elif visibility_fn is not None:
            vis = np.asarray(visibility_fn(qp, kpos), dtype=bool)
            visible = visible & _head_mask(vis, hq, end - start, nk)
        scores = np.where(visible, scores, -np.inf)
        row_any = visible.any(-1, keepdims=True)
        scores = np.where(row_any, scores, 0)
        m = scores.max(-1, keepdims=True)
        with np.errstate(invalid="ignore"):
            w = np.exp(scores - m)
        w = np.where(visible, w, 0)
        denom = w.sum(-1, keepdims=True)
        prob = np.where(row_any, w / np.where(denom == 0, 1, denom), 0).astype(a)
        rows = end - start
        pv = np.matmul(prob.reshape(hkv, group * rows, nk), values)
        outs.append(pv.reshape(hq, rows, -1).transpose(1, 0, 2))
        if return_positions:
            traces.append(positions)
    out = np.concatenate(outs, 0) if outs else np.zeros((0, hq, v.shape[2]), a)
    if return_positions:
        return out, np.concatenate(traces, 1)
    return out


def validate_contextual_path(positions, qpos, kpos, *, mask=None, atol=1e-6):
    """position.py:28-114 -- structural CoPE path checks on causal cells.

    Returns the reference's error message for the first failing check, or None.
    """
    positions = np.asarray(positions)
    if not np.isfinite(positions).all():
        return "positions must be finite floating [head,query,key]"
    dt = positions.dtype.type
    eps = dt(np.finfo(positions.dtype).eps)
    valid = np.broadcast_to(causal_mask(qpos, kpos)[None], positions.shape)
    if mask is not None:
        valid = valid & _head_mask(mask, *positions.shape)
    rounding = eps * np.abs(positions)
    tol = (dt(atol) + rounding).astype(dt)
    if ((positions < -tol) & valid).any():
        return NONNEGATIVE
    avail = (qpos[:, None] - kpos[None, :]).astype(dt)
    avail = np.maximum(avail, dt(-1)) + dt(1)
    if ((positions > (avail[None] + dt(atol) + rounding).astype(dt)) & valid).any():
        return AVAILABLE
    pairs = valid[..., :-1] & valid[..., 1:]
    diff = (positions[..., :-1] - positions[..., 1:]).astype(dt)
    gaps = (kpos[1:] - kpos[:-1]).astype(dt)
    ptol = (dt(atol) + rounding[..., :-1] + rounding[..., 1:]).astype(dt)
    if ((diff < -ptol) & pairs).any():
        return NONINCREASING
    if ((diff > gaps + ptol) & pairs).any():
        return ONE_GATE
    return None


def association_mask(qpos, kpos, fixed_indices, selected) -> np.ndarray:
    """attention.py:65-72 -- selected queries see non-fixed keys and themselves."""
    qpos, kpos = np.asarray(qpos), np.asarray(kpos)
    sel = np.isin(qpos, np.asarray(selected, dtype=np.int64))
    fixed_k = np.isin(kpos, np.asarray(fixed_indices, dtype=np.int64))
    return (~sel[:, None]) | (~fixed_k[None, :]) | (qpos[:, None] == kpos[None, :])


def canonical_transform(fixed_indices, table, table_rows, strict=False):
    """attention.py:32-57 -- substitute fixed x fixed cells from a canonical
    ``table [H, R, F]``; ``table_rows[ordinal]`` names the table row of each
    fixed query ordinal (profile lookup, position.py:701-748).  Returns a
    positions transform; with ``strict`` it also runs the path validation and
    raises ValueError with the reference's message.
    """
    ordinal = {int(p): i for i, p in enumerate(fixed_indices)}

    def transform(contextual, queries, keys):
        rows = [i for i, p in enumerate(queries.tolist()) if p in ordinal]
        if not rows:
            return contextual
        cols = [j for j, p in enumerate(keys.tolist()) if p in ordinal]
        ords = [ordinal[int(keys[j])] for j in cols]
        result = contextual.copy()
        for r in rows:
            trow = table_rows[ordinal[int(queries[r])]]
            result[:, r, cols] = table[:, trow, ords]
        if strict:
            message = validate_contextual_path(result, queries, keys)
            if message:
                raise ValueError(message)
        return result

    return transform


def ccpe_segments(fixed_indices, chunk_lengths, n: int):
    """The segments of an n-token prompt: each fixed chunk (``chunk_lengths``
    consecutive entries of ``fixed_indices``, contiguous in the prompt) and each
    maximal run of dynamic tokens, numbered in prompt order.  Returns
    (key_seg[n], seg_of_chunk[f], last_key[f], last_ord[f], ordinal[n]) with
    ordinal = the token's index in ``fixed_indices`` or -1 (the ordinal map
    of CanonicalPositionPolicy, attention.py:32-57)."""
    fixed_indices = np.asarray(fixed_indices, dtype=np.int64)
    ordinal = np.full(n, -1, dtype=np.int64)
    ordinal[fixed_indices] = np.arange(fixed_indices.size)
    chunk_of = np.full(n, -1, dtype=np.int64)
    ends = np.cumsum(chunk_lengths)
    starts = ends - np.asarray(chunk_lengths)
    for f, (a, b) in enumerate(zip(starts, ends)):
        chunk_of[fixed_indices[a:b]] = f
    key_seg = np.zeros(n, dtype=np.int64)
    seg = -1
    for t in range(n):
        if t == 0 or chunk_of[t] != chunk_of[t - 1] or (chunk_of[t] < 0) != (chunk_of[t - 1] < 0):
            seg += 1
        key_seg[t] = seg
    last_key = fixed_indices[ends - 1]
    return key_seg, key_seg[last_key], last_key, ends - 1, ordinal


def chunk_offsets_from_table(q, k, qpos, q_ord, q_seg, last_key, last_ord, seg_of_chunk,
                             table, n: int, nseg: int) -> np.ndarray:
    """Per-chunk carried counts from a canonical CCPE table (the compressed
    form of the CCPEProfile tables, position.py:581-748): for a fixed query
    row r and a fixed chunk f older than the query's segment, the table's
    position of the chunk's last key minus that key's gate
    sigmoid(q . k / sqrt(d)) in float32 (position.py:157-164); -1 elsewhere
    (the running count is carried).  Rows of tokens that are not queries stay
    -1 here."""
    H, d = q.shape[1], q.shape[2]
    G = H // k.shape[1]
    out = np.full((H, n, nseg), -1.0, dtype=np.float32)
    q32, k32 = q.astype(np.float32), k.astype(np.float32)
    inv = np.float32(1.0) / np.float32(np.sqrt(np.float32(d)))
    for r in range(q.shape[0]):
        if q_ord[r] < 0:
            continue
        for f in range(len(last_key)):
            if seg_of_chunk[f] >= q_seg[r]:
                continue
            kk = k32[last_key[f], np.arange(H) // G]                   # [H, d]
            logit = np.einsum("hd,hd->h", q32[r], kk).astype(np.float32) * inv
            gate = (np.float32(1) / (np.float32(1) + np.exp(-logit))).astype(np.float32)
            out[:, qpos[r], seg_of_chunk[f]] = table[:, q_ord[r], last_ord[f]] - gate
    return out
