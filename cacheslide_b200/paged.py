"""SLIDE indirection over the native paged KV cache (reference ``paged.py``).

``NativePagedKV`` keeps the reference's API and slot semantics; its device
work is the CUDA SLIDE kernels (``cs_slide_scatter`` / ``cs_slide_gather``)
over the caller's cache view ``[block, kv_head, block_offset, 2*D]``, which
may be non-contiguous (all four strides are honoured; nothing is reshaped or
copied).  Selected rows that are relocated live in a lazily allocated sidecar.

Beyond the reference it exposes ``device_view()`` and ``slot_table()``, with
which the attention kernel reads K/V straight through the slot map instead of
gathering a dense copy each step.
"""

from __future__ import annotations

import ctypes
import threading
from collections.abc import Iterable, Sequence
from concurrent.futures import Future

import torch

from . import _native as N
from .errors import StaleCompletionError  # noqa: F401  (re-exported for callers)
from .slide import LayerSlotMap, SlotWrite


def _indices(value: Sequence[int] | torch.Tensor, name: str) -> list[int]:
    """paged.py:21-32."""
    if isinstance(value, torch.Tensor):
        if value.ndim != 1 or value.dtype not in (torch.int32, torch.int64):
            raise ValueError(f"{name} must be an integer vector")
        value = value.detach().cpu().tolist()
    result = list(value)
    if any(type(item) is not int or item < 0 for item in result):
        raise ValueError(f"{name} must contain nonnegative integer positions")
    if len(set(result)) != len(result):
        raise ValueError(f"{name} must contain distinct positions")
    return result


def _completion_future(device: torch.device) -> Future:
    """Publish only after the device has executed the enqueued copies
    (paged.py:35-54): a CUDA event waited on by a daemon thread."""
    completed: Future = Future()
    completed.set_running_or_notify_cancel()
    if device.type != "cuda":
        completed.set_result(None)
        return completed
    event = torch.cuda.Event()
    event.record(torch.cuda.current_stream(device))

    def finish() -> None:
        try:
            event.synchronize()
        except BaseException as error:  # pragma: no cover - device failure path
            completed.set_exception(error)
        else:
            completed.set_result(None)

    threading.Thread(target=finish, name="cacheslide-kv-write", daemon=True).start()
    return completed


class NativePagedKV:
    """One request/layer's native slots plus its selected-token sidecar.

    See reference paged.py:57-581 for the contract; block ownership and pool
    capacity stay with the caller (vLLM), which may extend the block table
    through ``update_block_table`` before decode crosses a block boundary.
    """

    def __init__(
        self,
        cache: torch.Tensor,
        block_table: Sequence[int] | torch.Tensor,
        prompt_length: int,
        max_selected: int,
        *,
        request_id: str = "",
        layer_index: int = 0,
        shared_slots: Iterable[int] = (),
    ):
        if (
            not isinstance(cache, torch.Tensor)
            or cache.ndim != 4
            or min(cache.shape) < 1
            or cache.shape[-1] % 2
            or cache.dtype not in N.DTYPES
        ):
            raise ValueError("cache must be floating [blocks,KV heads,block size,2*D]")
        if cache.device.type != "cuda":
            raise ValueError("NativePagedKV runs on CUDA caches only (no CPU fallback)")
        if type(prompt_length) is not int or prompt_length < 1:
            raise ValueError("prompt_length must be a positive integer")
        if type(max_selected) is not int or max_selected < 0:
            raise ValueError("max_selected must be a nonnegative integer")
        if type(layer_index) is not int or layer_index < 0:
            raise ValueError("layer_index must be a nonnegative integer")
        self.cache = cache
        self.prompt_length = prompt_length
        self.request_id = request_id
        self.layer_index = layer_index
        self.block_size = cache.shape[2]
        self.kv_heads = cache.shape[1]
        self.head_dim = cache.shape[3] // 2
        self.native_total_slots = cache.shape[0] * self.block_size
        self.max_selected = max_selected
        self._mutex = threading.RLock()
        self._block_table = self._table(block_table)
        self._canonical = {t: self._canonical_slot(t) for t in range(prompt_length)}
        if len(set(self._canonical.values())) != prompt_length:
            raise ValueError("active logical blocks must name distinct native slots")
        self._shared = set(shared_slots)
        self.slot_map = LayerSlotMap(
            self._canonical,
            shared_slots=self._shared,
            allocation_floor=self.native_total_slots,
            max_slots=self.native_total_slots + max_selected,
        )
        self._side_key: torch.Tensor | None = None
        self._side_value: torch.Tensor | None = None
        self._baseline_ready: set[int] = set()
        self._loads: list[Future] = []
        self._promotions: list[Future] = []
        self._selected: set[int] = set()
        self._decoded = False
        self._hole_reuses = 0
        self._native_binds = 0
        self._canonical_mirrors = 0
        self._ready_inplace_writes = 0

    # ------------------------------------------------------------ geometry
    def _table(self, block_table) -> tuple[int, ...]:
        if isinstance(block_table, torch.Tensor):
            if block_table.ndim != 1 or block_table.dtype not in (torch.int32, torch.int64):
                raise ValueError("block_table must be a one-dimensional integer row")
            block_table = block_table.detach().cpu().tolist()
        row = tuple(block_table)
        if not row or any(
            type(b) is not int or not -1 <= b < self.cache.shape[0] for b in row
        ):
            raise ValueError("block_table contains invalid native block IDs")
        return row

    def _canonical_slot(self, token: int, row: tuple[int, ...] | None = None) -> int:
        row = self._block_table if row is None else row
        block_index, offset = divmod(token, self.block_size)
        if block_index >= len(row) or row[block_index] < 0:
            raise ValueError("logical token has no caller-owned native block")
        return row[block_index] * self.block_size + offset

    def update_block_table(self, block_table) -> None:
        row = self._table(block_table)
        with self._mutex:
            self.slot_map.snapshot()
            if any(self._canonical_slot(t, row) != s for t, s in self._canonical.items()):
                raise ValueError("block-table update moved an existing native token")
            self._block_table = row

    def canonical_slot(self, token: int) -> int:
        if type(token) is not int or token < 0:
            raise ValueError("token must be a nonnegative integer")
        with self._mutex:
            self.slot_map.snapshot()
            return self._canonical_slot(token)

    # ------------------------------------------------------- device access
    def device_view(self) -> N.PagedKV:
        """C-ABI description of the cache view and sidecar."""
        return N.paged_view(self.cache, self._side_key, self._side_value)

    def slot_table(self, logical_positions) -> torch.Tensor:
        """Current physical slot of each token as a device int64 vector."""
        positions = _indices(logical_positions, "logical_positions")
        with self._mutex:
            mapping = self.slot_map.snapshot()
            return torch.tensor(
                [mapping[t] for t in positions], dtype=torch.int64, device=self.cache.device
            )

    def _ensure_sidecar(self) -> None:
        if self._side_key is None:
            shape = (self.max_selected, self.kv_heads, self.head_dim)
            self._side_key = self.cache.new_empty(shape)
            self._side_value = self.cache.new_empty(shape)

    def _records(self, positions: list[int], key, value):
        expected = (len(positions), self.kv_heads, self.head_dim)
        for t in (key, value):
            if (
                not isinstance(t, torch.Tensor)
                or tuple(t.shape) != expected
                or t.device != self.cache.device
                or t.dtype != self.cache.dtype
            ):
                raise ValueError("K/V must match cache device/dtype and [token,KV head,D]")
        return key, value

    def _write_slots(self, slots: list[int], key, value, rows: list[int] | None = None) -> None:
        """cs_slide_scatter: record of slots[i] = (key, value)[rows[i] or i]."""
        if not slots:
            return
        if any(s >= self.native_total_slots for s in slots):
            self._ensure_sidecar()
        device = self.cache.device
        k = key if key.stride(-1) == 1 else key.contiguous()
        v = value if value.stride(-1) == 1 else value.contiguous()
        if k.stride() != v.stride():
            k, v = k.contiguous(), v.contiguous()
        slot_t = torch.tensor(slots, dtype=torch.int64, device=device)
        row_t = None if rows is None else torch.tensor(rows, dtype=torch.int64, device=device)
        status = N.Status(device)
        kv = self.device_view()
        N.check(
            N.load().cs_slide_scatter(
                ctypes.byref(kv), slot_t.data_ptr(), N.ptr(row_t), len(slots), k.data_ptr(),
                v.data_ptr(), k.stride(0), k.stride(1), status.ptr, N.stream_of(device),
            ),
            "cs_slide_scatter",
        )
        if status.read() & N.ST_SLOT_RANGE:
            raise ValueError("slot outside the native cache and sidecar")

    def _check_loads(self, *, allow_pending: bool = False) -> None:
        for loading in self._loads:
            if not loading.done():
                if allow_pending:
                    continue
                raise RuntimeError("source KV load must complete before baseline/mirror writes")
            loading.result()

    def _check_promotions(self) -> None:
        for promotion in self._promotions:
            if not promotion.done():
                raise RuntimeError("selected writes must complete before updating them")
            promotion.result()

    # --------------------------------------------------------------- writes
    def write(self, logical_positions, key: torch.Tensor, value: torch.Tensor) -> None:
        """Load baseline KV into original native slots (paged.py:242-274)."""
        positions = _indices(logical_positions, "logical_positions")
        self._records(positions, key, value)
        with self._mutex:
            self.slot_map.snapshot()
            self._check_loads()
            if self._decoded:
                raise RuntimeError("baseline writes cannot overwrite slots after decode")
            if any(t not in self._canonical for t in positions):
                raise KeyError("baseline writes require existing logical tokens")
            slots = [self._canonical[t] for t in positions]
            if self._shared.intersection(slots):
                raise ValueError("baseline writes cannot mutate shared native slots")
            with self.slot_map.write_guard(slots):
                try:
                    self._write_slots(slots, key, value)
                    _completion_future(self.cache.device).result()
                except BaseException:
                    self.slot_map.invalidate()
                    raise
            self._baseline_ready.update(positions)

    load_baseline = write

    def write_prefill(self, key: torch.Tensor, value: torch.Tensor) -> None:
        self.write(range(self.prompt_length), key, value)

    def promote_selected(
        self, logical_positions, key, value, *, load_future: Future | None = None
    ) -> Future:
        """Stage selected KV in the sidecar while a baseline load is pending."""
        positions = _indices(logical_positions, "logical_positions")
        self._records(positions, key, value)
        if load_future is not None and not isinstance(load_future, Future):
            raise TypeError("load_future must be a concurrent Future")
        with self._mutex:
            if self._decoded:
                raise RuntimeError("selected promotion must precede decode")
            if self._selected.intersection(positions):
                raise ValueError("already staged tokens must use update_selected")
            if load_future is not None and load_future.done():
                load_future.result()

            def writer(runs: list[SlotWrite]) -> Future:
                slots, rows = [], []
                for run in runs:
                    for i in range(run.slot_count):
                        slots.append(run.start_slot + i)
                        rows.append(int.from_bytes(run.payload[8 * i : 8 * i + 8], "little"))
                self._write_slots(slots, key, value, rows)
                return _completion_future(self.cache.device)

            # 8-byte payloads name tensor rows: no KV bytes leave the device
            updates = {t: row.to_bytes(8, "little") for row, t in enumerate(positions)}
            promotion = self.slot_map.promote_selected(
                updates, writer, load_future=load_future, allow_inplace=False
            )
            self._selected.update(positions)
            self._promotions.append(promotion)
            if load_future is not None and load_future not in self._loads:
                self._loads.append(load_future)
            return promotion

    stage_selected = promote_selected

    def write_selected_ready(self, logical_positions, key, value) -> dict[int, int]:
        """Load-first branch: overwrite original native slots in place."""
        positions = _indices(logical_positions, "logical_positions")
        self._records(positions, key, value)
        with self._mutex:
            mapping = self.slot_map.snapshot()
            self._check_loads()
            self._check_promotions()
            if self._decoded:
                raise RuntimeError("ready selected writes must precede decode")
            if len(self._baseline_ready) != self.prompt_length:
                raise RuntimeError("native baseline device writes must complete first")
            if not set(positions) <= set(self._canonical):
                raise ValueError("ready selected tokens require original native slots")
            if self._selected.intersection(positions) or any(
                mapping[t] != self._canonical[t] for t in positions
            ):
                raise ValueError("already selected tokens must use update_selected")
            slots = [self._canonical[t] for t in positions]
            with self.slot_map.write_guard(slots):
                try:
                    self._write_slots(slots, key, value)
                    _completion_future(self.cache.device).result()
                except BaseException:
                    self.slot_map.invalidate()
                    raise
            self._selected.update(positions)
            self._ready_inplace_writes += len(positions)
            return self.slot_map.snapshot()

    def _update_targets(self, positions: list[int]):
        """Current slots and the canonical mirrors worth attempting."""
        mapping = self.slot_map.snapshot()
        if not set(positions) <= set(mapping):
            raise ValueError("updated rows must already have logical mappings")
        if any(mapping[t] in self._shared for t in positions):
            raise ValueError("updated rows cannot mutate shared native slots")
        mirrors = [
            row
            for row, t in enumerate(positions)
            if self._canonical[t] not in self._shared and self._canonical[t] != mapping[t]
        ]
        return [mapping[t] for t in positions], mirrors

    def update_selected(self, logical_positions, key, value) -> None:
        """Write fused selected / fresh mandatory rows to their current slots,
        mirroring relocated rows into unpinned canonical slots."""
        positions = _indices(logical_positions, "logical_positions")
        self._records(positions, key, value)
        with self._mutex:
            self._check_loads()
            self._check_promotions()
            if self._decoded:
                raise RuntimeError("selected updates must precede decode hole reuse")
            slots, mirrors = self._update_targets(positions)
            optional = [self._canonical[positions[r]] for r in mirrors]
            with self.slot_map.write_guard(slots, optional_slots=optional) as writable:
                mirror_rows = [r for r in mirrors if self._canonical[positions[r]] in writable]
                try:
                    # one scatter for the current slots plus the mirrors
                    all_slots = slots + [self._canonical[positions[r]] for r in mirror_rows]
                    rows = list(range(len(slots))) + mirror_rows
                    self._write_slots(all_slots, key, value, rows)
                    _completion_future(self.cache.device).result()
                except BaseException:
                    self.slot_map.invalidate()
                    raise
                self._canonical_mirrors += len(mirror_rows)

    def update_fused(self, logical_positions, wca_state, layer_index, cached_k, cached_v,
                     recomputed_k, recomputed_v):
        """WCA update with the blend and the paged writes fused in one kernel.

        Equivalent to ``wca_state.update(...)`` followed by
        ``update_selected(positions, fused_k, fused_v)`` when no canonical
        mirror is needed (every row still maps to its own canonical slot);
        otherwise the mirrors are written by a second scatter.
        """
        positions = _indices(logical_positions, "logical_positions")
        with self._mutex:
            self._check_loads()
            self._check_promotions()
            if self._decoded:
                raise RuntimeError("selected updates must precede decode hole reuse")
            slots, mirrors = self._update_targets(positions)
            optional = [self._canonical[positions[r]] for r in mirrors]
            slot_t = torch.tensor(slots, dtype=torch.int64, device=self.cache.device)
            if any(s >= self.native_total_slots for s in slots):
                self._ensure_sidecar()
            with self.slot_map.write_guard(slots, optional_slots=optional) as writable:
                try:
                    update = wca_state.update(
                        layer_index, cached_k, cached_v, recomputed_k, recomputed_v,
                        computed_indices=torch.tensor(positions, device=self.cache.device),
                        paged=(self, slot_t),
                    )
                    mirror_rows = [r for r in mirrors if self._canonical[positions[r]] in writable]
                    if mirror_rows:
                        self._write_slots(
                            [self._canonical[positions[r]] for r in mirror_rows],
                            update.fused_k, update.fused_v, mirror_rows,
                        )
                    _completion_future(self.cache.device).result()
                except BaseException:
                    self.slot_map.invalidate()
                    raise
                self._canonical_mirrors += len(mirror_rows)
            return update

    # ---------------------------------------------------------------- reads
    def gather(self, logical_positions) -> tuple[torch.Tensor, torch.Tensor]:
        """Gather logical KV in caller order with atomic mapping pins."""
        positions = _indices(logical_positions, "logical_positions")
        with self._mutex, self.slot_map.pinned_mapping(positions) as mapping:
            self._check_loads(allow_pending=True)
            shape = (len(positions), self.kv_heads, self.head_dim)
            key, value = self.cache.new_empty(shape), self.cache.new_empty(shape)
            if positions:
                device = self.cache.device
                slot_t = torch.tensor(
                    [mapping[t] for t in positions], dtype=torch.int64, device=device
                )
                status = N.Status(device)
                kv = self.device_view()
                N.check(
                    N.load().cs_slide_gather(
                        ctypes.byref(kv), slot_t.data_ptr(), len(positions), key.data_ptr(),
                        value.data_ptr(), key.stride(0), key.stride(1), status.ptr,
                        N.stream_of(device),
                    ),
                    "cs_slide_gather",
                )
                if status.read() & N.ST_SLOT_RANGE:
                    raise ValueError("slot outside the native cache and sidecar")
            _completion_future(self.cache.device).result()
            return key, value

    # --------------------------------------------------------------- decode
    def decode(self, token: int, key, value, canonical_slot: int | None = None) -> int:
        """Reuse an eligible native hole, else bind the caller's slot; mirror."""
        if type(token) is not int or token < 0:
            raise ValueError("decode token must be a nonnegative integer")
        if key.ndim == 2:
            key = key.unsqueeze(0)
        if value.ndim == 2:
            value = value.unsqueeze(0)
        self._records([token], key, value)
        with self._mutex:
            self._check_loads(allow_pending=True)
            self._check_promotions()
            if token != len(self._canonical):
                raise ValueError("decode must append the next logical token")
            expected = self._canonical_slot(token)
            if canonical_slot is None:
                canonical_slot = expected
            if type(canonical_slot) is not int or canonical_slot != expected:
                raise ValueError("decode canonical slot is not owned by its block table")
            if canonical_slot in self._canonical.values():
                raise ValueError("decode native slot aliases an existing canonical token")
            with self.slot_map.decode_write_guard(
                token, canonical_slot, reuse_vacated=True
            ) as chosen:
                targets = [chosen] if chosen == canonical_slot else [chosen, canonical_slot]
                self._write_slots(targets, key, value, [0] * len(targets))
                _completion_future(self.cache.device).result()
            reused = chosen != canonical_slot
            self._hole_reuses += int(reused)
            self._canonical_mirrors += int(reused)
            self._native_binds += int(not reused)
            self._canonical[token] = canonical_slot
            self._decoded = True
            return chosen

    # ------------------------------------------------------------- metadata
    def snapshot(self) -> dict[int, int]:
        with self._mutex:
            return self.slot_map.snapshot()

    def page_metadata(self) -> tuple[dict[str, int | bool], ...]:
        with self._mutex:
            return self.slot_map.page_metadata(self.block_size, self._selected)

    def spill_order(self) -> tuple[int, ...]:
        """Advisory clean-first, most-selected-first page order (paged.py:540-559)."""
        pages = [p for p in self.page_metadata() if p["spill_eligible"]]
        pages.sort(key=lambda p: (p["dirty"], -p["selected_count"], p["page_id"]))
        return tuple(p["page_id"] for p in pages)

    def stats(self) -> dict[str, int]:
        with self._mutex:
            return {
                **self.slot_map.stats(),
                "physical_hole_reuse": self._hole_reuses,
                "decode_native_bind": self._native_binds,
                "canonical_mirror_writes": self._canonical_mirrors,
                "sidecar_capacity_slots": self.max_selected,
                "sidecar_allocated_slots": (
                    self.max_selected if self._side_key is not None else 0
                ),
                "selected_ready_inplace_writes": self._ready_inplace_writes,
                "native_pool_capacity_slots": self.native_total_slots,
                "native_pool_capacity_blocks": self.cache.shape[0],
                "native_pool_capacity_delta": 0,
                "native_pool_blocks_released": 0,
            }

    def invalidate(self) -> None:
        with self._mutex:
            self.slot_map.invalidate()
