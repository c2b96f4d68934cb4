"""Contextual position encoding (CoPE) and CCPE attention on B200.

Drop-in for the reference module ``cacheslide_vllm.position``: same names,
argument meaning and exception types (``CCPEPositionError`` for invalid
substituted paths, ``ValueError`` for shape/schema problems).  All arithmetic
runs in CUDA kernels of ``libcacheslide_sm100.so``; CPU tensors are rejected.

Mode selection of :func:`cope_attention` (reference position.py:404-560):

* plain CoPE, ``attention_mask``, ``visibility_mask``, ``fixed_positions`` and
  the known policies (:class:`~cacheslide_b200.attention.CanonicalPositionPolicy`,
  :class:`~cacheslide_b200.attention.SelectedAssociationPolicy`,
  :class:`ChunkResetPositions`) run inside one attention launch;
* any other ``positions_transform`` / ``visibility_transform`` callable keeps
  the reference's per-query-chunk contract: the kernel first emits the chunk's
  contextual positions, the callable transforms them, and a second launch
  attends with the transformed positions.

The reference's training-only pieces (autograd, ``position_trace`` and
``CCPEProfile.calibrate``) are offline calibration and are not part of this
reuse-time package.
"""

from __future__ import annotations

import ctypes
import math
import re
from collections.abc import Callable
from dataclasses import dataclass

import torch
from torch import Tensor, nn

from . import _native as N


class CCPEPositionError(ValueError):
    """A canonical substitution does not define a valid contextual path."""


_PATH_MESSAGES = (
    (N.ST_PATH_NEG, "causal contextual positions must be nonnegative"),
    (N.ST_PATH_AVAIL, "causal contextual count exceeds available gates"),
    (N.ST_PATH_INCR, "causal contextual path must be nonincreasing"),
    (N.ST_PATH_GAP, "causal contextual path exceeds one gate per token"),
)


def path_error(bits: int) -> str | None:
    """Reference message of the first failing path check (position.py:99-114)."""
    for bit, message in _PATH_MESSAGES:
        if bits & bit:
            return message
    return None


def _accumulation_dtype(tensor: Tensor) -> torch.dtype:
    """position.py:153-154."""
    return torch.float64 if tensor.dtype == torch.float64 else torch.float32


def _all_finite(t: Tensor) -> bool:
    return bool(torch.isfinite(t).all())


def _rows(name: str, tensor: Tensor) -> None:
    """position.py:117-124."""
    if (
        not isinstance(tensor, Tensor)
        or tensor.ndim != 3
        or not tensor.is_floating_point()
        or min(tensor.shape[1:]) < 1
        or not _all_finite(tensor)
    ):
        raise ValueError(f"{name} must be finite floating [token, head, dimension]")


def _positions(name: str, tensor: Tensor, n: int, device: torch.device) -> None:
    """position.py:127-137."""
    if (
        not isinstance(tensor, Tensor)
        or tensor.ndim != 1
        or tensor.shape[0] != n
        or tensor.dtype != torch.long
        or tensor.device != device
        or bool((tensor < 0).any())
    ):
        raise ValueError(f"{name} must be nonnegative int64 [{n}] on {device}")
    if torch.unique(tensor).numel() != n:
        raise ValueError(f"{name} must identify distinct token positions")


def _qk_layout(query: Tensor, key: Tensor) -> None:
    """position.py:140-150."""
    _rows("query", query)
    _rows("key", key)
    if query.device != key.device or query.dtype != key.dtype:
        raise ValueError("Q/K dtype and device must match")
    if query.shape[-1] != key.shape[-1]:
        raise ValueError("Q/K head dimensions must match")
    if query.shape[1] % key.shape[1]:
        raise ValueError("query heads must be a multiple of KV heads for GQA")
    if key.shape[0] == 0:
        raise ValueError("attention requires at least one key")


def _increasing(key_positions: Tensor) -> bool:
    return key_positions.numel() <= 1 or bool((key_positions[1:] > key_positions[:-1]).all())


def _mask_u8(mask: Tensor, heads: int, nq: int, nk: int) -> tuple[Tensor, int, int]:
    """bool mask [q,k] | [1,q,k] | [h,q,k] -> uint8 view + (h stride, q stride)."""
    m = mask
    if m.ndim == 2:
        m = m.unsqueeze(0)
    m = m.to(torch.uint8)
    if m.stride(-1) != 1:
        m = m.contiguous()
    sh = 0 if m.shape[0] == 1 else m.stride(0)
    return m, sh, m.stride(1)


def validate_contextual_path(
    positions: Tensor,
    query_positions: Tensor,
    key_positions: Tensor,
    *,
    attention_mask: Tensor | None = None,
    atol: float = 1e-6,
) -> None:
    """Structural CoPE path checks (position.py:28-114) in one CUDA launch."""
    if (
        not isinstance(positions, Tensor)
        or positions.ndim != 3
        or not positions.is_floating_point()
        or positions.shape[0] < 1
        or positions.shape[2] < 1
    ):
        raise CCPEPositionError("positions must be finite floating [head,query,key]")
    if isinstance(atol, bool) or not isinstance(atol, (int, float)) or not math.isfinite(atol) \
            or atol < 0:
        raise CCPEPositionError("atol must be finite and nonnegative")
    device = N.require_cuda(positions)
    for name, coordinates, size in (
        ("query_positions", query_positions, positions.shape[1]),
        ("key_positions", key_positions, positions.shape[2]),
    ):
        if not isinstance(coordinates, Tensor):
            raise CCPEPositionError(f"{name} must be an int64 tensor")
        try:
            _positions(name, coordinates, size, device)
        except ValueError as error:
            raise CCPEPositionError(str(error)) from error
    if not _increasing(key_positions):
        raise CCPEPositionError("key_positions must be strictly increasing")
    mask, msh, msq = None, 0, 0
    if attention_mask is not None:
        if (
            not isinstance(attention_mask, Tensor)
            or attention_mask.dtype != torch.bool
            or attention_mask.device != device
            or attention_mask.shape
            not in (positions.shape[1:], (1, *positions.shape[1:]), positions.shape)
        ):
            raise CCPEPositionError(
                "attention_mask must be bool [query,key] or [head,query,key]"
            )
        mask, msh, msq = _mask_u8(attention_mask, *positions.shape)
    pos = positions
    dt = N.CS_F64 if pos.dtype == torch.float64 else N.CS_F32
    if pos.dtype not in (torch.float32, torch.float64):
        pos = pos.float()
    if pos.stride(-1) != 1:
        pos = pos.contiguous()
    qpos, kpos = query_positions.contiguous(), key_positions.contiguous()
    status = N.Status(device)
    N.check(
        N.load().cs_cope_validate_path(
            pos.data_ptr(), pos.stride(0), pos.stride(1), qpos.data_ptr(), kpos.data_ptr(),
            N.ptr(mask), msh, msq, pos.shape[0], pos.shape[1], pos.shape[2], float(atol), dt,
            status.ptr, N.stream_of(device),
        ),
        "validate_contextual_path",
    )
    bits = status.read()
    if bits & N.ST_POS_RANGE:
        raise CCPEPositionError("positions must be finite floating [head,query,key]")
    message = path_error(bits)
    if message:
        raise CCPEPositionError(message)


class CoPE(nn.Module):
    """Learned contextual bias shared across heads; embeddings [dim, max_positions].

    Mirrors ``cacheslide_vllm.position.CoPE`` (position.py:275-367) for
    reuse-time inference; every method dispatches to a CUDA kernel.
    """

    def __init__(
        self,
        head_dim: int,
        max_positions: int,
        *,
        device: torch.device | str | None = None,
        dtype: torch.dtype | None = None,
    ) -> None:
        super().__init__()
        if head_dim < 1 or max_positions < 2:
            raise ValueError("head_dim must be positive and max_positions at least two")
        self.head_dim = head_dim
        self.max_positions = max_positions
        self.position_embeddings = nn.Parameter(
            torch.zeros(head_dim, max_positions, device=device, dtype=dtype),
            requires_grad=False,
        )

    def contextual_positions(self, logits: Tensor, allowed_mask: Tensor) -> Tensor:
        """Mask before sigmoid, reverse-cumsum over causal keys, then clamp."""
        if logits.ndim != 3 or not logits.is_floating_point():
            raise ValueError("logits must be floating [head,query,key]")
        if allowed_mask.shape != logits.shape or allowed_mask.dtype != torch.bool:
            raise ValueError("allowed_mask must be bool with the logits shape")
        if allowed_mask.device != logits.device:
            raise ValueError("allowed_mask and logits must share a device")
        device = N.require_cuda(logits)
        acc = torch.float64 if logits.dtype == torch.float64 else torch.float32
        lg = logits.to(acc)
        if lg.stride(-1) != 1:
            lg = lg.contiguous()
        allowed = allowed_mask.to(torch.uint8)
        if allowed.stride(-1) != 1:
            allowed = allowed.contiguous()
        out = torch.empty(logits.shape, dtype=acc, device=device)
        status = N.Status(device)
        N.check(
            N.load().cs_cope_positions(
                lg.data_ptr(), lg.stride(0), lg.stride(1), allowed.data_ptr(), allowed.stride(0),
                allowed.stride(1), lg.shape[0], lg.shape[1], lg.shape[2], self.max_positions,
                N.CS_F64 if acc == torch.float64 else N.CS_F32, out.data_ptr(), out.stride(0),
                out.stride(1), status.ptr, N.stream_of(device),
            ),
            "contextual_positions",
        )
        if status.read() & N.ST_LOGIT_NONFINITE:
            raise ValueError("unmasked logits must be finite")
        return out.to(logits.dtype)

    def positional_bias(self, query: Tensor, positions: Tensor) -> Tensor:
        """Interpolate between floor(p) and its clamped right-hand neighbour."""
        _rows("query", query)
        if query.shape[-1] != self.head_dim:
            raise ValueError("query dimension does not match the learned embeddings")
        if query.device != self.position_embeddings.device:
            raise ValueError("query and learned embeddings must share a device")
        if (
            positions.ndim != 3
            or positions.shape[:2] != (query.shape[1], query.shape[0])
            or not positions.is_floating_point()
            or positions.device != query.device
        ):
            raise ValueError("positions must be bounded query-dependent [head,query,key]")
        device = N.require_cuda(query)
        acc = _accumulation_dtype(query)
        q = query if query.stride(-1) == 1 else query.contiguous()
        E = self.position_embeddings.detach().to(acc)
        pos = positions.to(acc)
        if pos.stride(-1) != 1:
            pos = pos.contiguous()
        out = torch.empty(positions.shape, dtype=acc, device=device)
        status = N.Status(device)
        N.check(
            N.load().cs_cope_bias(
                q.data_ptr(), q.stride(0), q.stride(1), E.data_ptr(), E.stride(0), E.stride(1),
                self.head_dim, self.max_positions, pos.data_ptr(), pos.stride(0), pos.stride(1),
                q.shape[1], q.shape[0], pos.shape[2], N.DTYPES[q.dtype], out.data_ptr(),
                out.stride(0), out.stride(1), status.ptr, N.stream_of(device),
            ),
            "positional_bias",
        )
        if status.read() & N.ST_POS_RANGE:
            raise ValueError("positions must be bounded query-dependent [head,query,key]")
        return out

    def forward(
        self,
        query: Tensor,
        key: Tensor,
        query_positions: Tensor,
        key_positions: Tensor | None = None,
        *,
        attention_mask: Tensor | None = None,
        fixed_positions: Tensor | None = None,
    ) -> Tensor:
        """Bias [head, query, key] from contextual (or fixed) positions."""
        _qk_layout(query, key)
        device = N.require_cuda(query, key)
        _positions("query_positions", query_positions, query.shape[0], device)
        if key_positions is None:
            key_positions = torch.arange(key.shape[0], device=device)
        _positions("key_positions", key_positions, key.shape[0], device)
        if not _increasing(key_positions):
            raise ValueError("key_positions must be strictly increasing for reverse cumsum")
        if fixed_positions is None:
            positions = _kernel_positions(
                query, key, self, query_positions, key_positions, attention_mask
            )
        else:
            positions = fixed_positions
        if positions.shape != (query.shape[1], query.shape[0], key.shape[0]):
            raise ValueError("fixed_positions must exactly match [head,query,key]")
        return self.positional_bias(query, positions)


@dataclass(frozen=True)
class ChunkIdentity:
    """One reusable chunk of an ordered CCPE layout (position.py:563-577)."""

    role: str
    content_hash: str
    length: int

    def __post_init__(self) -> None:
        if not self.role.strip() or not re.fullmatch(r"[0-9a-f]{64}", self.content_hash):
            raise ValueError("chunk needs a nonempty role and lowercase SHA-256 hash")
        if not isinstance(self.length, int) or isinstance(self.length, bool):
            raise ValueError("chunk length must be a positive integer")
        if self.length <= 0:
            raise ValueError("chunk length must be a positive integer")


@dataclass(frozen=True)
class ChunkResetPositions:
    """Compressed CCPE positions: reverse gate counts restart at chunk boundaries.

    ``key_chunk[j]`` (int, nondecreasing over keys) names the chunk of key j;
    ``offsets[h, t, c]`` (float32, indexed by query token position t) is the
    canonical count carried into chunk ``c`` from the newer chunks, for chunks
    older than the query's own chunk.  A negative offset carries the actual
    running count (no reset), so all-negative offsets give plain CoPE.  This
    replaces the quadratic ``[head, F, F]`` canonical tables of
    ``CCPEProfile`` (position.py:581-748) with a per-chunk representation.
    """

    key_chunk: Tensor
    offsets: Tensor

    def __call__(self, contextual: Tensor, queries: Tensor, keys: Tensor) -> Tensor:
        raise RuntimeError(
            "ChunkResetPositions is evaluated inside the attention kernel; "
            "pass it as cope_attention(positions_transform=...)"
        )

    @classmethod
    def from_profile(
        cls,
        table: Tensor,
        fixed_indices,
        chunk_lengths,
        num_tokens: int,
        query: Tensor,
        query_positions: Tensor,
        key: Tensor,
        *,
        table_query_positions: Tensor | None = None,
    ) -> ChunkResetPositions:
        """The compressed form of a canonical CCPE table for one prompt.

        ``table`` is a CCPEProfile's ``canonical_positions`` ``[head, Fq, F]``
        (position.py:581-748): row ``i`` holds fixed query ordinal
        ``table_query_positions[i]`` (default ``i``), column ``j`` fixed key
        ordinal ``j``.  ``fixed_indices`` are the prompt positions of the fixed
        tokens in order and ``chunk_lengths`` the lengths of the fixed chunks
        (a plan's ``fixed_indices`` and ``fixed_layout``, attention.py:32-57);
        ``query`` ``[nq, hq, d]`` at ``query_positions`` and ``key``
        ``[num_tokens, hkv, d]`` are the prompt's current rows.

        The prompt is cut into segments -- each fixed chunk and each run of
        dynamic tokens -- and for a fixed query and a fixed chunk older than
        the query's segment the offset is the carried count into the chunk:
        the table's position of the chunk's last key minus that key's gate
        (``cs_cope_chunk_offsets``, on the device).  Inside the fixed chunks
        the kernels then recount the current gates, so with the calibration's
        fixed content every fixed x fixed position equals its table entry;
        dynamic keys carry the running count.
        """
        device = N.require_cuda(query)
        n = int(num_tokens)
        lengths = [int(x) for x in chunk_lengths]
        fixed = [int(x) for x in fixed_indices]
        if sum(lengths) != len(fixed) or any(x <= 0 for x in lengths):
            raise ValueError("fixed chunk lengths must be positive and cover fixed_indices")
        if any(b <= a for a, b in zip(fixed, fixed[1:])) or (fixed and not 0 <= fixed[0] <= fixed[-1] < n):
            raise ValueError("fixed_indices must be increasing positions inside the prompt")
        if query.ndim != 3 or key.ndim != 3 or key.shape[0] != n:
            raise ValueError("query must be [nq, hq, d] and key [num_tokens, hkv, d]")
        if query.dtype != key.dtype or query.dtype not in (torch.float32, torch.float16,
                                                          torch.bfloat16):
            raise ValueError("query and key must share a float32 / float16 / bfloat16 dtype")
        hq, d, hkv = query.shape[1], query.shape[2], key.shape[1]
        if key.shape[2] != d or hq % hkv:
            raise ValueError("query / key heads or head dims do not match")
        if table.ndim != 3 or table.shape[0] != hq or table.shape[2] != len(fixed):
            raise ValueError("table must be [query heads, profiled rows, fixed keys]")
        # segments: fixed chunks and dynamic runs, in prompt order
        chunk_of = [-1] * n
        start = 0
        for f, length in enumerate(lengths):
            for pos in fixed[start:start + length]:
                chunk_of[pos] = f
            start += length
        key_seg, seg = [], -1
        for t in range(n):
            if t == 0 or chunk_of[t] != chunk_of[t - 1]:
                seg += 1
            key_seg.append(seg)
        nseg = seg + 1
        ends = [sum(lengths[:f + 1]) for f in range(len(lengths))]
        last_key = [fixed[e - 1] for e in ends]
        last_ord = [e - 1 for e in ends]
        seg_of_chunk = [key_seg[t] for t in last_key]
        ordinal = {pos: i for i, pos in enumerate(fixed)}
        if table_query_positions is None:
            rows = {i: i for i in range(table.shape[1])}
        else:
            rows = {int(o): i for i, o in enumerate(table_query_positions.tolist())}
        qpos = [int(x) for x in query_positions.tolist()]
        if len(qpos) != query.shape[0] or any(not 0 <= t < n for t in qpos):
            raise ValueError("query_positions must give one prompt position per query row")
        q_ord = []
        for t in qpos:
            o = ordinal.get(t, -1)
            if o >= 0 and o not in rows:
                raise ValueError("CCPE profile has no contextual trace for these query positions")
            q_ord.append(rows[o] if o >= 0 else -1)
        i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=device)  # noqa: E731
        qpos_t = torch.tensor(qpos, dtype=torch.int64, device=device)
        tab = table.to(device=device, dtype=torch.float32)
        offsets = torch.full((hq, n, nseg), -1.0, dtype=torch.float32, device=device)
        args = dict(q_ord=i32(q_ord), q_seg=i32([key_seg[t] for t in qpos]),
                    last_key=torch.tensor(last_key, dtype=torch.int64, device=device),
                    last_ord=i32(last_ord), seg_of_chunk=i32(seg_of_chunk))
        status = N.Status(device)
        N.check(N.load().cs_cope_chunk_offsets(
            query.data_ptr(), query.stride(0), query.stride(1), query.shape[0], hq, d,
            qpos_t.data_ptr(), args["q_ord"].data_ptr(), args["q_seg"].data_ptr(),
            key.data_ptr(), key.stride(0), key.stride(1), hkv, args["last_key"].data_ptr(),
            args["last_ord"].data_ptr(), args["seg_of_chunk"].data_ptr(), len(lengths),
            tab.data_ptr(), tab.stride(0), tab.stride(1), tab.stride(2), tab.shape[1],
            tab.shape[2], N.DTYPES[query.dtype], offsets.data_ptr(), offsets.stride(0),
            offsets.stride(1), nseg, status.ptr, N.stream_of(device)), "cs_cope_chunk_offsets")
        if status.read():
            raise ValueError("table ordinals out of range")
        return cls(key_chunk=i32(key_seg), offsets=offsets)


def _base_params(
    query: Tensor,
    key: Tensor | None,
    value: Tensor | None,
    cope: CoPE,
    qpos: Tensor,
    kpos: Tensor | None,
    nk: int,
    hkv: int,
    dv: int,
) -> N.AttnParams:
    p = N.AttnParams()
    p.q = query.data_ptr()
    p.q_stride_tok, p.q_stride_head = query.stride(0), query.stride(1)
    p.nq, p.hq, p.d = query.shape[0], query.shape[1], query.shape[2]
    p.qpos = qpos.data_ptr()
    if key is not None:
        p.k, p.v = key.data_ptr(), value.data_ptr()
        p.k_stride_tok, p.k_stride_head = key.stride(0), key.stride(1)
        p.v_stride_tok, p.v_stride_head = value.stride(0), value.stride(1)
    p.nk, p.hkv, p.dv = nk, hkv, dv
    p.kpos = N.ptr(kpos)
    E = cope.position_embeddings.detach()
    p.E = E.data_ptr()
    p.e_stride_d, p.e_stride_p = E.stride(0), E.stride(1)
    p.npos = cope.max_positions
    p.scale = math.sqrt(query.shape[-1])
    p.in_dtype = N.DTYPES[query.dtype]
    p.out_dtype = N.DTYPES[query.dtype]
    p.atol = 1e-6
    return p


DECODE_MAX_ROWS = 8  # split-key decode for at most this many query rows ...
DECODE_MIN_KEYS = 512  # ... over at least this many keys


def _launch(p: N.AttnParams, device: torch.device, *, allow_fast: bool) -> None:
    """Split-key decode for a few rows over a long context, the tensor-core
    prefill when the mode allows it, else the generic kernel."""
    lib = N.load()
    stream = N.stream_of(device)
    if allow_fast and p.nq <= DECODE_MAX_ROWS and p.nk >= DECODE_MIN_KEYS:
        size = lib.cs_cope_attn_decode_workspace(ctypes.byref(p))
        if size > 0:
            workspace = torch.empty(size, dtype=torch.uint8, device=device)
            N.check(lib.cs_cope_attn_decode(ctypes.byref(p), workspace.data_ptr(), stream),
                    "cs_cope_attn_decode")
            return
    if allow_fast:
        rc = lib.cs_cope_attn_prefill(ctypes.byref(p), stream)
        if rc == N.CS_OK:
            return
        if rc != N.CS_ERR_UNSUPPORTED:
            N.check(rc, "cs_cope_attn_prefill")
    N.check(lib.cs_cope_attn(ctypes.byref(p), stream), "cs_cope_attn")


def _kernel_positions(query, key, cope, qpos, kpos, attention_mask) -> Tensor:
    """Contextual positions [h, q, k] from the attention kernel's scan."""
    device = query.device
    acc = _accumulation_dtype(query)
    E = cope.position_embeddings.detach().to(acc)
    holder = _Holder(cope, E)
    q = query if query.stride(-1) == 1 else query.contiguous()
    k = key if key.stride(-1) == 1 else key.contiguous()
    out = torch.zeros((q.shape[1], q.shape[0], k.shape[0]), dtype=acc, device=device)
    p = _base_params(q, k, k, holder, qpos, kpos, k.shape[0], k.shape[1], k.shape[2])
    p.positions_only = 1
    p.out_positions = out.data_ptr()
    p.op_stride_h, p.op_stride_q = out.stride(0), out.stride(1)
    gm = None
    if attention_mask is not None:
        gm, p.gm_stride_h, p.gm_stride_q = _mask_u8(attention_mask, *out.shape)
        p.gate_mask = gm.data_ptr()
    status = N.Status(device)
    p.status = status.ptr
    _launch(p, device, allow_fast=False)
    bits = status.read()
    if bits & (N.ST_LOGIT_NONFINITE | N.ST_INPUT_NONFINITE):
        raise ValueError("attention logits overflowed the accumulation dtype")
    return out


class _Holder:
    """CoPE stand-in whose table is in the accumulation dtype, as the kernels
    read it (the reference upcasts E, position.py:335-338)."""

    def __init__(self, cope: CoPE, E: Tensor):
        self.position_embeddings = E
        self.max_positions = cope.max_positions
        self.head_dim = cope.head_dim


def cope_attention(
    query: Tensor,
    key: Tensor,
    value: Tensor,
    cope: CoPE,
    query_positions: Tensor,
    key_positions: Tensor | None = None,
    *,
    attention_mask: Tensor | None = None,
    visibility_mask: Tensor | None = None,
    fixed_positions: Tensor | None = None,
    positions_transform: Callable[[Tensor, Tensor, Tensor], Tensor] | None = None,
    visibility_transform: Callable[[Tensor, Tensor], Tensor] | None = None,
    query_chunk_size: int = 128,
    return_positions: bool = False,
) -> Tensor | tuple[Tensor, Tensor]:
    """CoPE/CCPE attention (reference position.py:404-560) on the GPU.

    Order of operations: causal gates, position transform, learned bias,
    visibility transform, masked softmax (fully masked rows give zero), PV,
    cast to ``value.dtype``.  ``query_chunk_size`` bounds only the working set
    of generic callable transforms; kernel-side modes process all rows at once.
    """
    from .attention import CanonicalPositionPolicy, SelectedAssociationPolicy

    _qk_layout(query, key)
    _rows("value", value)
    if value.shape[:2] != key.shape[:2] or value.device != key.device or \
            value.dtype != key.dtype:
        raise ValueError("K/V token count, heads, dtype and device must match")
    if not isinstance(query_chunk_size, int) or query_chunk_size < 1:
        raise ValueError("query_chunk_size must be a positive integer")
    if positions_transform is not None:
        if not callable(positions_transform):
            raise CCPEPositionError("positions_transform must be callable")
        if fixed_positions is not None:
            raise CCPEPositionError(
                "positions_transform and fixed_positions are mutually exclusive"
            )
    if visibility_transform is not None:
        if not callable(visibility_transform):
            raise ValueError("visibility_transform must be callable")
        if visibility_mask is not None:
            raise ValueError("visibility_transform and visibility_mask are mutually exclusive")
    device = N.require_cuda(query, key, value)
    _positions("query_positions", query_positions, query.shape[0], device)
    if key_positions is None:
        key_positions = torch.arange(key.shape[0], device=device)
    _positions("key_positions", key_positions, key.shape[0], device)
    if not _increasing(key_positions):
        raise ValueError("key_positions must be strictly increasing for reverse cumsum")
    nq, hq, nk = query.shape[0], query.shape[1], key.shape[0]
    for name, mask in (("attention_mask", attention_mask), ("visibility_mask", visibility_mask)):
        if mask is not None and mask.shape not in ((nq, nk), (1, nq, nk), (hq, nq, nk)):
            raise ValueError(f"{name} has an incompatible full-query shape")
        if mask is not None and (mask.dtype != torch.bool or mask.device != device):
            raise ValueError(f"{name} must be bool on the query device")
    acc = _accumulation_dtype(query)
    if fixed_positions is not None:
        if fixed_positions.shape != (hq, nq, nk):
            raise ValueError("fixed_positions must be full query-dependent [head,query,key]")
        if (
            not fixed_positions.is_floating_point()
            or fixed_positions.device != device
            or not _all_finite(fixed_positions)
            or bool((fixed_positions < 0).any())
            or bool((fixed_positions > cope.max_positions - 1).any())
        ):
            raise ValueError("positions must be bounded query-dependent [head,query,key]")
    if query.shape[-1] != cope.head_dim or cope.position_embeddings.device != device:
        raise ValueError("query and learned embeddings must share a device and dimension")

    q = query if query.stride(-1) == 1 else query.contiguous()
    k = key if key.stride(-1) == 1 else key.contiguous()
    v = value if value.stride(-1) == 1 else value.contiguous()
    qpos = query_positions.contiguous()
    kpos = key_positions.contiguous()
    E = cope.position_embeddings.detach().to(acc)
    holder = _Holder(cope, E)
    out = torch.empty((nq, hq, v.shape[2]), dtype=value.dtype, device=device)
    trace = None
    if return_positions:
        trace = torch.zeros((hq, nq, nk), dtype=acc, device=device)
    if nq == 0:
        return (out, trace) if return_positions else out

    keep = []  # tensors whose pointers the launch uses

    def params(rows: slice) -> N.AttnParams:
        qs = q[rows]
        p = _base_params(qs, k, v, holder, qpos[rows], kpos, nk, k.shape[1], v.shape[2])
        p.out = out[rows].data_ptr()
        p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
        p.out_dtype = N.DTYPES[value.dtype]
        if attention_mask is not None:
            gm, p.gm_stride_h, p.gm_stride_q = _mask_u8(attention_mask, hq, nq, nk)
            keep.append(gm)
            p.gate_mask = gm[:, rows].data_ptr()
        if trace is not None:
            p.out_positions = trace[:, rows].data_ptr()
            p.op_stride_h, p.op_stride_q = trace.stride(0), trace.stride(1)
        return p

    assoc = None
    if isinstance(visibility_transform, SelectedAssociationPolicy):
        assoc = visibility_transform.flags(qpos, kpos)
    vis_fn = None if (assoc is not None or visibility_transform is None) else visibility_transform

    known_pos = positions_transform is None or isinstance(
        positions_transform, (CanonicalPositionPolicy, ChunkResetPositions)
    )
    status = N.Status(device)

    if known_pos and vis_fn is None:
        p = params(slice(0, nq))
        p.status = status.ptr
        if visibility_mask is not None:
            vm, p.vm_stride_h, p.vm_stride_q = _mask_u8(visibility_mask, hq, nq, nk)
            keep.append(vm)
            p.vis_mask = vm.data_ptr()
        if assoc is not None:
            keep.extend(assoc)
            p.q_selected, p.k_fixed = assoc[0].data_ptr(), assoc[1].data_ptr()
        if fixed_positions is not None:
            fp = fixed_positions.to(acc)
            keep.append(fp)
            p.pos_mode = N.POS_FIXED
            p.fixed_pos = fp.data_ptr()
            p.fp_stride_h, p.fp_stride_q, p.fp_stride_k = fp.stride()
        elif isinstance(positions_transform, CanonicalPositionPolicy):
            keep.extend(positions_transform.bind(p, qpos, kpos, acc, device))
        elif isinstance(positions_transform, ChunkResetPositions):
            keep.extend(_bind_chunk_reset(p, positions_transform, qpos, kpos, hq, device))
        fast = (
            p.pos_mode in (N.POS_CONTEXTUAL, N.POS_CHUNK, N.POS_TABLE)
            and attention_mask is None
            and visibility_mask is None
            and trace is None
        )
        _launch(p, device, allow_fast=fast)
        _raise_status(status.read(), strict=bool(p.strict))
    else:
        # generic callables: per query chunk, positions -> transform -> attend
        for start in range(0, nq, query_chunk_size):
            rows = slice(start, min(start + query_chunk_size, nq))
            qp = qpos[rows]
            if positions_transform is not None:
                pos = torch.zeros((hq, rows.stop - start, nk), dtype=acc, device=device)
                pp = params(rows)
                pp.positions_only = 1
                pp.out_positions = pos.data_ptr()
                pp.op_stride_h, pp.op_stride_q = pos.stride(0), pos.stride(1)
                st = N.Status(device)
                pp.status = st.ptr
                _launch(pp, device, allow_fast=False)
                _raise_status(st.read(), strict=False)
                if isinstance(positions_transform, CanonicalPositionPolicy):
                    transformed = positions_transform(pos, qp, kpos)
                else:
                    transformed = positions_transform(pos, qp, kpos)
                if (
                    not isinstance(transformed, Tensor)
                    or transformed.shape != pos.shape
                    or transformed.dtype != pos.dtype
                    or transformed.device != pos.device
                    or not _all_finite(transformed)
                    or bool((transformed < 0).any())
                    or bool((transformed > cope.max_positions - 1).any())
                ):
                    raise CCPEPositionError(
                        "positions_transform must return bounded finite positions "
                        "with the contextual shape, dtype and device"
                    )
            p = params(rows)
            st = N.Status(device)
            p.status = st.ptr
            if positions_transform is not None:
                tp = transformed.contiguous()
                keep.append(tp)
                p.pos_mode = N.POS_FIXED
                p.fixed_pos = tp.data_ptr()
                p.fp_stride_h, p.fp_stride_q, p.fp_stride_k = tp.stride()
                if trace is not None:
                    trace[:, rows] = transformed
                    p.out_positions = None
            elif fixed_positions is not None:
                fp = fixed_positions.to(acc)[:, rows].contiguous()
                keep.append(fp)
                p.pos_mode = N.POS_FIXED
                p.fixed_pos = fp.data_ptr()
                p.fp_stride_h, p.fp_stride_q, p.fp_stride_k = fp.stride()
            vis = None
            if visibility_mask is not None:
                vis = visibility_mask[..., rows, :]
            elif vis_fn is not None:
                vis = vis_fn(qp, kpos)
                if not isinstance(vis, Tensor):
                    raise ValueError("visibility_transform must return a bool tensor")
                if vis.dtype != torch.bool or vis.device != device or vis.shape not in (
                    (rows.stop - start, nk), (1, rows.stop - start, nk),
                    (hq, rows.stop - start, nk),
                ):
                    raise ValueError("attention_mask must be [query,key] or [head,query,key]")
            if vis is not None:
                vm, p.vm_stride_h, p.vm_stride_q = _mask_u8(vis, hq, rows.stop - start, nk)
                keep.append(vm)
                p.vis_mask = vm.data_ptr()
            if assoc is not None:
                p.q_selected = assoc[0][rows].data_ptr()
                p.k_fixed = assoc[1].data_ptr()
            _launch(p, device, allow_fast=False)
            _raise_status(st.read(), strict=False)
    del keep
    return (out, trace) if return_positions else out


def _raise_status(bits: int, *, strict: bool) -> None:
    if bits & N.ST_SLOT_RANGE:
        raise ValueError("paged KV slot outside the arena")
    if strict:
        message = path_error(bits)
        if message:
            raise CCPEPositionError(message)
    if bits & N.ST_POS_RANGE:
        raise CCPEPositionError(
            "positions_transform must return bounded finite positions "
            "with the contextual shape, dtype and device"
        )
    if bits & (N.ST_LOGIT_NONFINITE | N.ST_INPUT_NONFINITE):
        raise ValueError("contextual attention logits are not finite")


def _bind_chunk_reset(p, policy: ChunkResetPositions, qpos, kpos, hq, device):
    key_chunk = policy.key_chunk.to(device=device, dtype=torch.int32).contiguous()
    if key_chunk.shape != (p.nk,):
        raise ValueError("key_chunk must name the chunk of every key")
    if key_chunk.numel() > 1 and bool((key_chunk[1:] < key_chunk[:-1]).any()):
        raise ValueError("key_chunk must be nondecreasing over keys")
    offsets = policy.offsets
    if offsets.ndim != 3 or offsets.shape[0] != hq:
        raise ValueError("chunk offsets must be [head, token, chunk]")
    nchunks = int(key_chunk.max().item()) + 1 if key_chunk.numel() else 1
    if offsets.shape[2] < nchunks:
        raise ValueError("chunk offsets must cover every key chunk")
    rows = offsets.to(device=device, dtype=torch.float32).index_select(1, qpos).contiguous()
    p.pos_mode = N.POS_CHUNK
    p.key_chunk = key_chunk.data_ptr()
    p.chunk_off = rows.data_ptr()
    p.co_stride_h, p.co_stride_q = rows.stride(0), rows.stride(1)
    p.nchunks = offsets.shape[2]
    return [key_chunk, rows]
