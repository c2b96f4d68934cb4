"""CCPE coordinate and WCA visibility policies (reference ``attention.py``).

Both policies keep the reference's call contract, so they can be called on a
query tile directly.  When passed to :func:`cacheslide_b200.position.cope_attention`
they are not called per tile: ``bind``/``flags`` turn them into the kernel's
canonical-table mode and association flags, evaluated inside the attention
launch.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
from torch import Tensor

from . import _native as N
from .position import ChunkIdentity, validate_contextual_path


def _chunk_identities(plan, profile) -> tuple:
    """Ordered fixed layout as the profile's own ChunkIdentity type, so that a
    profile calibrated by either package compares equal (position.py:721)."""
    chunks = getattr(profile, "chunks", None)
    kind = type(chunks[0]) if chunks else ChunkIdentity
    return tuple(kind(*entry) for entry in plan.fixed_layout)


@dataclass(frozen=True)
class CanonicalPositionPolicy:
    """Substitute fixed x fixed cells with canonical profile positions.

    reference attention.py:18-57.  ``mode="strict_contextual"`` validates the
    hybrid path and raises ``CCPEPositionError``; ``"mixed_bias_override"``
    accepts it.
    """

    plan: object
    profile: object
    checkpoint_id: str
    mode: str = "strict_contextual"

    def __post_init__(self):
        if not isinstance(self.mode, str) or self.mode not in {
            "strict_contextual",
            "mixed_bias_override",
        }:
            raise ValueError("unknown CCPE position policy")

    def _ordinals(self) -> dict[int, int]:
        return {position: i for i, position in enumerate(self.plan.fixed_indices)}

    def _lookup(self, ordinals: list[int], device, dtype) -> Tensor:
        return self.profile.lookup(
            _chunk_identities(self.plan, self.profile),
            torch.tensor(ordinals, dtype=torch.long),
            checkpoint_id=self.checkpoint_id,
            trained_profile_version=self.profile.trained_profile_version,
            device=device,
            dtype=dtype,
        )

    def __call__(self, contextual: Tensor, queries: Tensor, keys: Tensor) -> Tensor:
        ordinal = self._ordinals()
        rows = [i for i, p in enumerate(queries.tolist()) if p in ordinal]
        if not rows:
            return contextual
        canonical = self._lookup(
            [ordinal[int(queries[i])] for i in rows], contextual.device, contextual.dtype
        )
        columns = [i for i, p in enumerate(keys.tolist()) if p in ordinal]
        fixed_ordinals = [ordinal[int(keys[i])] for i in columns]
        result = contextual.clone()
        r = torch.tensor(rows, device=contextual.device)
        c = torch.tensor(columns, device=contextual.device, dtype=torch.long)
        o = torch.tensor(fixed_ordinals, device=contextual.device, dtype=torch.long)
        result[:, r[:, None], c[None, :]] = canonical[:, :, o]
        if self.mode == "strict_contextual":
            validate_contextual_path(result, queries, keys)
        return result

    def bind(self, p: N.AttnParams, qpos: Tensor, kpos: Tensor, acc, device) -> list[Tensor]:
        """Configure the kernel's canonical-table mode for these rows/keys.

        ``q_row[i]`` indexes the looked-up table rows of fixed queries (-1 for
        dynamic ones), ``k_ord[j]`` is the fixed ordinal of key j (-1 for
        dynamic keys); the kernel then substitutes table[h, q_row, k_ord].
        """
        ordinal = self._ordinals()
        qlist = qpos.tolist()
        rows = [i for i, pos in enumerate(qlist) if pos in ordinal]
        if not rows:
            return []
        table = self._lookup([ordinal[qlist[i]] for i in rows], device, acc).contiguous()
        if not bool(torch.isfinite(table).all()) or bool((table < 0).any()) or bool(
            (table > p.npos - 1).any()
        ):
            from .position import CCPEPositionError

            raise CCPEPositionError(
                "positions_transform must return bounded finite positions "
                "with the contextual shape, dtype and device"
            )
        q_row = [-1] * len(qlist)
        for r, i in enumerate(rows):
            q_row[i] = r
        k_ord = [ordinal.get(pos, -1) for pos in kpos.tolist()]
        q_row_t = torch.tensor(q_row, dtype=torch.int32, device=device)
        k_ord_t = torch.tensor(k_ord, dtype=torch.int32, device=device)
        p.pos_mode = N.POS_TABLE
        p.table = table.data_ptr()
        p.tb_stride_h, p.tb_stride_r, p.tb_stride_c = table.stride()
        p.q_row, p.k_ord = q_row_t.data_ptr(), k_ord_t.data_ptr()
        p.strict = 1 if self.mode == "strict_contextual" else 0
        return [table, q_row_t, k_ord_t]


@dataclass(frozen=True)
class SelectedAssociationPolicy:
    """WCA association after gate counting (reference attention.py:60-72):
    selected queries see only non-fixed keys plus themselves."""

    fixed_indices: tuple[int, ...]
    selected_indices: Tensor

    def __call__(self, queries: Tensor, keys: Tensor) -> Tensor:
        fixed = torch.tensor(self.fixed_indices, device=keys.device, dtype=torch.long)
        selected = torch.isin(queries, self.selected_indices.to(queries.device))
        return (
            ~selected[:, None]
            | ~torch.isin(keys, fixed)[None, :]
            | (queries[:, None] == keys[None, :])
        )

    def flags(self, qpos: Tensor, kpos: Tensor) -> tuple[Tensor, Tensor]:
        """Per-query `selected` and per-key `fixed` bytes for the kernel."""
        fixed = torch.tensor(self.fixed_indices, device=kpos.device, dtype=torch.long)
        q_sel = torch.isin(qpos, self.selected_indices.to(qpos.device)).to(torch.uint8)
        k_fix = torch.isin(kpos, fixed).to(torch.uint8)
        return q_sel.contiguous(), k_fix.contiguous()
