"""SLIDE indirection over the caller's native paged KV cache.

Public contract (``src/cacheslide_vllm/paged.py:57-581``): ``NativePagedKV``
with the reference's constructor, methods, slot choices, statistics and error
messages, so a runtime written against the reference switches without edits.
The implementation is this module's own:

* tensor data moves only through the CUDA SLIDE kernels
  (``cs_slide_scatter`` / ``cs_slide_gather``) over the caller's view
  ``[block, kv_head, block_offset, 2*D]`` with all four strides honoured
  (nothing is reshaped or copied); relocated rows live in a sidecar that is
  allocated on the first relocation;
* every device write or read is enqueued together with an asynchronous copy
  of its status word into pinned host memory and a CUDA event, so one event
  wait gives both completion and the kernel's status (``_Launch``);
* asynchronous completions (a promotion whose mapping is published when its
  copies have run) are resolved by one shared waiter thread per process that
  takes events in order (``_Waiter``), not a thread per write;
* the canonical (block-table) slot of each token is a list indexed by token.

Beyond the reference it exposes ``device_view()`` and ``slot_table()``, with
which the attention kernels read K/V through the slot map instead of
gathering a dense copy every step.
"""

from __future__ import annotations

import ctypes
import queue
import threading
from collections.abc import Iterable, Sequence
from concurrent.futures import Future
from dataclasses import dataclass

import torch

from . import _native as N
from .errors import StaleCompletionError  # noqa: F401  (re-exported for callers)
from .slide import LayerSlotMap, SlotWrite

_ROW_BYTES = 8  # a promotion record names a row of the caller's K/V tensors


def _positions(value: Sequence[int] | torch.Tensor, name: str) -> list[int]:
    """Distinct nonnegative token positions from a list or an integer vector
    (the reference's argument contract, paged.py:21-32)."""
    if isinstance(value, torch.Tensor):
        if value.ndim != 1 or value.dtype not in (torch.int32, torch.int64):
            raise ValueError(f"{name} must be an integer vector")
        value = value.detach().cpu().tolist()
    out = list(value)
    for item in out:
        if type(item) is not int or item < 0:
            raise ValueError(f"{name} must contain nonnegative integer positions")
    if len(set(out)) != len(out):
        raise ValueError(f"{name} must contain distinct positions")
    return out


class _Launch:
    """A device operation in flight: its event and its status word, copied to
    pinned host memory behind the kernel on the same stream."""

    def __init__(self, device: torch.device):
        self.device = device
        self.word = torch.zeros(1, dtype=torch.int32, device=device)
        self.host = torch.empty(1, dtype=torch.int32, pin_memory=True)
        self.event = torch.cuda.Event()

    @property
    def status_ptr(self) -> int:
        return self.word.data_ptr()

    def enqueue_done(self) -> "_Launch":
        stream = torch.cuda.current_stream(self.device)
        self.host.copy_(self.word, non_blocking=True)
        self.event.record(stream)
        return self

    def bits(self) -> int:
        """Status bits; valid once the event has completed."""
        return int(self.host[0])

    def check(self) -> None:
        if self.bits() & N.ST_SLOT_RANGE:
            raise ValueError("slot outside the native cache and sidecar")

    def wait(self) -> None:
        self.event.synchronize()
        self.check()


class _Waiter:
    """One daemon thread resolving futures when their launches complete."""

    _lock = threading.Lock()
    _queue: queue.SimpleQueue | None = None

    @classmethod
    def submit(cls, launch: _Launch) -> Future:
        done: Future = Future()
        done.set_running_or_notify_cancel()
        with cls._lock:
            if cls._queue is None:
                cls._queue = queue.SimpleQueue()
                threading.Thread(target=cls._run, args=(cls._queue,),
                                 name="cacheslide-kv-completion", daemon=True).start()
            cls._queue.put((launch, done))
        return done

    @staticmethod
    def _run(q: queue.SimpleQueue) -> None:
        while True:
            launch, done = q.get()
            try:
                launch.wait()
            except BaseException as error:  # device failure or bad slot
                done.set_exception(error)
            else:
                done.set_result(None)


@dataclass
class PageSpill:
    """Pages written back by ``NativePagedKV.spill``: page ids in spill order,
    their images ``[pages, kv_heads, block_size, 2 * head_dim]`` in pinned
    host memory, and a Future that completes when the copy has landed."""

    pages: tuple[int, ...]
    images: torch.Tensor
    future: Future


class NativePagedKV:
    """One request/layer's native slots plus its selected-token sidecar.

    Block ownership and pool capacity stay with the caller (vLLM): the arena
    writes only slots its block table names, never frees a block, and the
    caller extends the table through ``update_block_table`` before decode
    crosses a block boundary.  Once a selected row has been relocated,
    attention must read through this map (``gather`` or ``slot_table``).
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
        shape_ok = (isinstance(cache, torch.Tensor) and cache.ndim == 4
                    and min(cache.shape) >= 1 and cache.shape[-1] % 2 == 0
                    and cache.dtype in N.DTYPES)
        if not shape_ok:
            raise ValueError("cache must be floating [blocks,KV heads,block size,2*D]")
        if cache.device.type != "cuda":
            raise ValueError("NativePagedKV runs on CUDA caches only (no CPU fallback)")
        for name, value, low in (("prompt_length", prompt_length, 1),
                                 ("max_selected", max_selected, 0),
                                 ("layer_index", layer_index, 0)):
            if type(value) is not int or value < low:
                kind = "a positive" if low else "a nonnegative"
                raise ValueError(f"{name} must be {kind} integer")
        self.cache = cache
        self.prompt_length = prompt_length
        self.request_id = request_id
        self.layer_index = layer_index
        self.kv_heads = cache.shape[1]
        self.block_size = cache.shape[2]
        self.head_dim = cache.shape[3] // 2
        self.native_total_slots = cache.shape[0] * self.block_size
        self.max_selected = max_selected
        self._lock = threading.RLock()
        self._blocks = self._parse_table(block_table)
        self._home = [self._slot_in(self._blocks, t) for t in range(prompt_length)]
        self._home_set = set(self._home)
        if len(self._home_set) != prompt_length:
            raise ValueError("active logical blocks must name distinct native slots")
        self._shared = set(shared_slots)
        self.slot_map = LayerSlotMap(
            dict(enumerate(self._home)),
            shared_slots=self._shared,
            allocation_floor=self.native_total_slots,
            max_slots=self.native_total_slots + max_selected,
        )
        self._side_key: torch.Tensor | None = None
        self._side_value: torch.Tensor | None = None
        self._baseline = bytearray(prompt_length)  # 1 = device write completed
        self._baseline_count = 0
        self._loads: list[Future] = []
        self._promotions: list[Future] = []
        self._selected: set[int] = set()
        self._decoded = False
        self._counts = dict(hole_reuse=0, native_bind=0, mirrors=0, ready_inplace=0)

    # ------------------------------------------------------------ geometry
    def _parse_table(self, block_table) -> tuple[int, ...]:
        if isinstance(block_table, torch.Tensor):
            if block_table.ndim != 1 or block_table.dtype not in (torch.int32, torch.int64):
                raise ValueError("block_table must be a one-dimensional integer row")
            block_table = block_table.detach().cpu().tolist()
        row = tuple(block_table)
        limit = self.cache.shape[0]
        if not row or not all(type(b) is int and -1 <= b < limit for b in row):
            raise ValueError("block_table contains invalid native block IDs")
        return row

    def _slot_in(self, row: tuple[int, ...], token: int) -> int:
        block, offset = divmod(token, self.block_size)
        if block >= len(row) or row[block] < 0:
            raise ValueError("logical token has no caller-owned native block")
        return row[block] * self.block_size + offset

    def update_block_table(self, block_table) -> None:
        """Adopt a longer caller-owned table; existing tokens must not move."""
        row = self._parse_table(block_table)
        with self._lock:
            self.slot_map.snapshot()  # raises once retired
            for token, slot in enumerate(self._home):
                if self._slot_in(row, token) != slot:
                    raise ValueError("block-table update moved an existing native token")
            self._blocks = row

    def canonical_slot(self, token: int) -> int:
        if type(token) is not int or token < 0:
            raise ValueError("token must be a nonnegative integer")
        with self._lock:
            self.slot_map.snapshot()
            return self._slot_in(self._blocks, token)

    # ------------------------------------------------------- device access
    def device_view(self) -> N.PagedKV:
        """C-ABI description of the cache view and its sidecar."""
        return N.paged_view(self.cache, self._side_key, self._side_value)

    def slot_table(self, logical_positions) -> torch.Tensor:
        """Current physical slot of each token as a device int64 vector."""
        positions = _positions(logical_positions, "logical_positions")
        with self._lock:
            mapping = self.slot_map.snapshot()
            return torch.tensor([mapping[t] for t in positions], dtype=torch.int64,
                                device=self.cache.device)

    def _check_rows(self, count: int, key, value) -> None:
        want = (count, self.kv_heads, self.head_dim)
        for t in (key, value):
            if (not isinstance(t, torch.Tensor) or tuple(t.shape) != want
                    or t.device != self.cache.device or t.dtype != self.cache.dtype):
                raise ValueError("K/V must match cache device/dtype and [token,KV head,D]")

    def _scatter(self, slots: list[int], key, value, rows: list[int] | None = None) -> _Launch:
        """Enqueue record of slots[i] = (key, value)[rows[i] if rows else i]."""
        device = self.cache.device
        launch = _Launch(device)
        if not slots:
            return launch.enqueue_done()
        if self._side_key is None and max(slots) >= self.native_total_slots:
            shape = (self.max_selected, self.kv_heads, self.head_dim)
            self._side_key = self.cache.new_empty(shape)
            self._side_value = self.cache.new_empty(shape)
        k = key if key.stride(-1) == 1 else key.contiguous()
        v = value if value.stride(-1) == 1 else value.contiguous()
        if k.stride() != v.stride():
            k, v = k.contiguous(), v.contiguous()
        slot_t = torch.tensor(slots, dtype=torch.int64).to(device, non_blocking=True)
        row_t = (None if rows is None
                 else torch.tensor(rows, dtype=torch.int64).to(device, non_blocking=True))
        view = self.device_view()
        N.check(N.load().cs_slide_scatter(
            ctypes.byref(view), slot_t.data_ptr(), N.ptr(row_t), len(slots), k.data_ptr(),
            v.data_ptr(), k.stride(0), k.stride(1), launch.status_ptr, N.stream_of(device)),
            "cs_slide_scatter")
        return launch.enqueue_done()

    def _sync_write(self, slots: list[int], key, value, rows=None) -> None:
        with self.slot_map.write_guard(slots):
            try:
                self._scatter(slots, key, value, rows).wait()
            except BaseException:
                self.slot_map.invalidate()
                raise

    def _loads_settled(self, pending_ok: bool = False) -> None:
        for load in self._loads:
            if load.done():
                load.result()  # a failed load re-raises here
            elif not pending_ok:
                raise RuntimeError("source KV load must complete before baseline/mirror writes")

    def _promotions_settled(self) -> None:
        for promotion in self._promotions:
            if not promotion.done():
                raise RuntimeError("selected writes must complete before updating them")
            promotion.result()

    # --------------------------------------------------------------- writes
    def write(self, logical_positions, key: torch.Tensor, value: torch.Tensor) -> None:
        """Baseline KV into the tokens' own native slots, whatever the current
        redirection (paged.py:242-274); waits for the device write."""
        positions = _positions(logical_positions, "logical_positions")
        self._check_rows(len(positions), key, value)
        with self._lock:
            self.slot_map.snapshot()
            self._loads_settled()
            if self._decoded:
                raise RuntimeError("baseline writes cannot overwrite slots after decode")
            if any(t >= len(self._home) for t in positions):
                raise KeyError("baseline writes require existing logical tokens")
            slots = [self._home[t] for t in positions]
            if not self._shared.isdisjoint(slots):
                raise ValueError("baseline writes cannot mutate shared native slots")
            self._sync_write(slots, key, value)
            for t in positions:
                if t < self.prompt_length and not self._baseline[t]:
                    self._baseline[t] = 1
                    self._baseline_count += 1

    load_baseline = write

    def write_prefill(self, key: torch.Tensor, value: torch.Tensor) -> None:
        self.write(range(self.prompt_length), key, value)

    def promote_selected(self, logical_positions, key, value, *,
                         load_future: Future | None = None) -> Future:
        """Copy-on-write of selected rows into the sidecar while a baseline
        load may still be pending; the returned future resolves to the
        published map once the copies have run (paged.py:276-328)."""
        positions = _positions(logical_positions, "logical_positions")
        self._check_rows(len(positions), key, value)
        if load_future is not None and not isinstance(load_future, Future):
            raise TypeError("load_future must be a concurrent Future")
        with self._lock:
            if self._decoded:
                raise RuntimeError("selected promotion must precede decode")
            if not self._selected.isdisjoint(positions):
                raise ValueError("already staged tokens must use update_selected")
            if load_future is not None and load_future.done():
                load_future.result()

            def writer(runs: list[SlotWrite]) -> Future:
                slots, rows = [], []
                for run in runs:
                    for i in range(run.slot_count):
                        slots.append(run.start_slot + i)
                        rec = run.payload[i * _ROW_BYTES:(i + 1) * _ROW_BYTES]
                        rows.append(int.from_bytes(rec, "little"))
                return _Waiter.submit(self._scatter(slots, key, value, rows))

            # the records name rows of key/value; no KV byte leaves the device
            records = {t: row.to_bytes(_ROW_BYTES, "little") for row, t in enumerate(positions)}
            promotion = self.slot_map.promote_selected(
                records, writer, load_future=load_future, allow_inplace=False)
            self._selected.update(positions)
            self._promotions.append(promotion)
            if load_future is not None and all(f is not load_future for f in self._loads):
                self._loads.append(load_future)
            return promotion

    stage_selected = promote_selected

    def write_selected_ready(self, logical_positions, key, value) -> dict[int, int]:
        """Load-first branch: overwrite the selected tokens' own native slots
        once the whole baseline is on the device (paged.py:330-374)."""
        positions = _positions(logical_positions, "logical_positions")
        self._check_rows(len(positions), key, value)
        with self._lock:
            mapping = self.slot_map.snapshot()
            self._loads_settled()
            self._promotions_settled()
            if self._decoded:
                raise RuntimeError("ready selected writes must precede decode")
            if self._baseline_count != self.prompt_length:
                raise RuntimeError("native baseline device writes must complete first")
            if any(t >= len(self._home) for t in positions):
                raise ValueError("ready selected tokens require original native slots")
            moved = any(mapping[t] != self._home[t] for t in positions)
            if moved or not self._selected.isdisjoint(positions):
                raise ValueError("already selected tokens must use update_selected")
            self._sync_write([self._home[t] for t in positions], key, value)
            self._selected.update(positions)
            self._counts["ready_inplace"] += len(positions)
            return self.slot_map.snapshot()

    def _targets(self, positions: list[int]) -> tuple[list[int], list[int]]:
        """Current slots of the rows, and the rows whose own native slot is
        worth mirroring to (relocated and not shared)."""
        mapping = self.slot_map.snapshot()
        if any(t not in mapping for t in positions):
            raise ValueError("updated rows must already have logical mappings")
        current = [mapping[t] for t in positions]
        if not self._shared.isdisjoint(current):
            raise ValueError("updated rows cannot mutate shared native slots")
        mirrors = [r for r, t in enumerate(positions)
                   if self._home[t] != current[r] and self._home[t] not in self._shared]
        return current, mirrors

    def _ready_for_update(self) -> None:
        self._loads_settled()
        self._promotions_settled()
        if self._decoded:
            raise RuntimeError("selected updates must precede decode hole reuse")

    def update_selected(self, logical_positions, key, value) -> None:
        """Fused rows into their current slots, mirrored into their own native
        slots where those are free (paged.py:376-431); one scatter."""
        positions = _positions(logical_positions, "logical_positions")
        self._check_rows(len(positions), key, value)
        with self._lock:
            self._ready_for_update()
            current, mirrors = self._targets(positions)
            homes = [self._home[positions[r]] for r in mirrors]
            with self.slot_map.write_guard(current, optional_slots=homes) as free:
                mirror_rows = [r for r in mirrors if self._home[positions[r]] in free]
                slots = current + [self._home[positions[r]] for r in mirror_rows]
                rows = list(range(len(current))) + mirror_rows
                try:
                    self._scatter(slots, key, value, rows).wait()
                except BaseException:
                    self.slot_map.invalidate()
                    raise
                self._counts["mirrors"] += len(mirror_rows)

    def update_fused(self, logical_positions, wca_state, layer_index, cached_k, cached_v,
                     recomputed_k, recomputed_v):
        """``wca_state.update`` with the blend written straight into the rows'
        current paged slots by the same kernel, then the mirrors.  Equal to
        ``update`` followed by ``update_selected(positions, fused_k, fused_v)``."""
        positions = _positions(logical_positions, "logical_positions")
        with self._lock:
            self._ready_for_update()
            current, mirrors = self._targets(positions)
            homes = [self._home[positions[r]] for r in mirrors]
            slot_t = torch.tensor(current, dtype=torch.int64, device=self.cache.device)
            if self._side_key is None and current and max(current) >= self.native_total_slots:
                shape = (self.max_selected, self.kv_heads, self.head_dim)
                self._side_key = self.cache.new_empty(shape)
                self._side_value = self.cache.new_empty(shape)
            with self.slot_map.write_guard(current, optional_slots=homes) as free:
                try:
                    result = wca_state.update(
                        layer_index, cached_k, cached_v, recomputed_k, recomputed_v,
                        computed_indices=torch.tensor(positions, device=self.cache.device),
                        paged=(self, slot_t))
                    mirror_rows = [r for r in mirrors if self._home[positions[r]] in free]
                    self._scatter([self._home[positions[r]] for r in mirror_rows],
                                  result.fused_k, result.fused_v, mirror_rows).wait()
                except BaseException:
                    self.slot_map.invalidate()
                    raise
                self._counts["mirrors"] += len(mirror_rows)
            return result

    # ---------------------------------------------------------------- reads
    def gather(self, logical_positions) -> tuple[torch.Tensor, torch.Tensor]:
        """Logical KV in caller order; the mappings stay pinned until the
        device reads have completed (paged.py:433-472)."""
        positions = _positions(logical_positions, "logical_positions")
        with self._lock, self.slot_map.pinned_mapping(positions) as mapping:
            self._loads_settled(pending_ok=True)
            shape = (len(positions), self.kv_heads, self.head_dim)
            key, value = self.cache.new_empty(shape), self.cache.new_empty(shape)
            device = self.cache.device
            launch = _Launch(device)
            if positions:
                slot_t = torch.tensor([mapping[t] for t in positions],
                                      dtype=torch.int64).to(device, non_blocking=True)
                view = self.device_view()
                N.check(N.load().cs_slide_gather(
                    ctypes.byref(view), slot_t.data_ptr(), len(positions), key.data_ptr(),
                    value.data_ptr(), key.stride(0), key.stride(1), launch.status_ptr,
                    N.stream_of(device)), "cs_slide_gather")
            launch.enqueue_done().wait()
            return key, value

    # --------------------------------------------------------------- decode
    def decode(self, token: int, key, value, canonical_slot: int | None = None) -> int:
        """Append decode token ``token``: the lowest idle native hole if any,
        else the caller's native slot for it, plus a mirror into that slot
        when a hole was taken (paged.py:474-524).  Returns the slot chosen."""
        if type(token) is not int or token < 0:
            raise ValueError("decode token must be a nonnegative integer")
        key = key.unsqueeze(0) if key.ndim == 2 else key
        value = value.unsqueeze(0) if value.ndim == 2 else value
        self._check_rows(1, key, value)
        with self._lock:
            self._loads_settled(pending_ok=True)
            self._promotions_settled()
            if token != len(self._home):
                raise ValueError("decode must append the next logical token")
            own = self._slot_in(self._blocks, token)
            if canonical_slot is None:
                canonical_slot = own
            if type(canonical_slot) is not int or canonical_slot != own:
                raise ValueError("decode canonical slot is not owned by its block table")
            if canonical_slot in self._home_set:
                raise ValueError("decode native slot aliases an existing canonical token")
            with self.slot_map.decode_write_guard(token, canonical_slot,
                                                  reuse_vacated=True) as chosen:
                targets = sorted({chosen, canonical_slot})
                self._scatter(targets, key, value, [0] * len(targets)).wait()
            hole = chosen != canonical_slot
            self._counts["hole_reuse"] += hole
            self._counts["mirrors"] += hole
            self._counts["native_bind"] += not hole
            self._home.append(canonical_slot)
            self._home_set.add(canonical_slot)
            self._decoded = True
            return chosen

    # ------------------------------------------------------------- metadata
    def snapshot(self) -> dict[int, int]:
        with self._lock:
            return self.slot_map.snapshot()

    def page_metadata(self) -> tuple[dict[str, int | bool], ...]:
        """Per mapped physical page of this arena: token / selected counts
        and guards (``dirty`` = holds a selected token)."""
        with self._lock:
            return self.slot_map.page_metadata(self.block_size, self._selected)

    def spill_order(self) -> tuple[int, ...]:
        """Advisory page order for a spill (paged.py:530-559): guarded pages
        excluded, clean before dirty, then more selected tokens first, then
        page id.  Reserves nothing."""
        eligible = [p for p in self.page_metadata() if p["spill_eligible"]]
        ranked = sorted(eligible,
                        key=lambda p: (p["dirty"], -p["selected_count"], p["page_id"]))
        return tuple(p["page_id"] for p in ranked)

    def spill(self, pages: Sequence[int] | None = None) -> PageSpill:
        """Write back pages: their images (one native block each, the
        records of its ``block_size`` slots; ``cs_slide_pack_pages``) copied
        into pinned host memory.  ``pages`` defaults to ``spill_order()`` (the
        reference only advises that order, paged.py:530-559).  The pages'
        slots stay pinned until the host copy has landed, so no relocation or
        write lands in them meanwhile; the returned ``PageSpill`` carries the
        page ids, the host images and a Future of the copy."""
        with self._lock:
            ids = list(self.spill_order() if pages is None else pages)
            if any(type(p) is not int or p < 0 for p in ids) or len(set(ids)) != len(ids):
                raise ValueError("pages must be distinct nonnegative page ids")
            bs = self.block_size
            slots = [p * bs + o for p in ids for o in range(bs)]
            mapped = set(self.slot_map.snapshot().values())
            guard = self.slot_map.pin_slots([x for x in slots if x in mapped])
            guard.__enter__()
            try:
                device = self.cache.device
                shape = (len(ids), self.kv_heads, bs, 2 * self.head_dim)
                image = self.cache.new_empty(shape)
                host = torch.empty(shape, dtype=self.cache.dtype, pin_memory=True)
                launch = _Launch(device)
                if ids:
                    page_t = torch.tensor(ids, dtype=torch.int64).to(device, non_blocking=True)
                    view = self.device_view()
                    N.check(N.load().cs_slide_pack_pages(
                        ctypes.byref(view), page_t.data_ptr(), len(ids), image.data_ptr(),
                        launch.status_ptr, N.stream_of(device)), "cs_slide_pack_pages")
                    host.copy_(image, non_blocking=True)
                future = _Waiter.submit(launch.enqueue_done())
            except BaseException:
                guard.__exit__(None, None, None)
                raise
            # the pins end when the copy has landed (or failed)
            future.add_done_callback(lambda _f: guard.__exit__(None, None, None))
            return PageSpill(tuple(ids), host, future)

    def reload(self, spilled: PageSpill) -> None:
        """Write a spill's page images back into the same pages
        (``cs_slide_unpack_pages``), with the slots' write guards held until
        the device writes complete."""
        with self._lock:
            spilled.future.result()
            ids = list(spilled.pages)
            bs = self.block_size
            slots = [p * bs + o for p in ids for o in range(bs)]
            mapped = set(self.slot_map.snapshot().values())
            with self.slot_map.write_guard([x for x in slots if x in mapped]):
                device = self.cache.device
                launch = _Launch(device)
                if ids:
                    image = spilled.images.to(device, non_blocking=True)
                    page_t = torch.tensor(ids, dtype=torch.int64).to(device, non_blocking=True)
                    view = self.device_view()
                    N.check(N.load().cs_slide_unpack_pages(
                        ctypes.byref(view), page_t.data_ptr(), len(ids), image.data_ptr(),
                        launch.status_ptr, N.stream_of(device)), "cs_slide_unpack_pages")
                launch.enqueue_done().wait()

    def stats(self) -> dict[str, int]:
        with self._lock:
            c = self._counts
            return {
                **self.slot_map.stats(),
                "physical_hole_reuse": c["hole_reuse"],
                "decode_native_bind": c["native_bind"],
                "canonical_mirror_writes": c["mirrors"],
                "sidecar_capacity_slots": self.max_selected,
                "sidecar_allocated_slots": 0 if self._side_key is None else self.max_selected,
                "selected_ready_inplace_writes": c["ready_inplace"],
                "native_pool_capacity_slots": self.native_total_slots,
                "native_pool_capacity_blocks": self.cache.shape[0],
                "native_pool_capacity_delta": 0,
                "native_pool_blocks_released": 0,
            }

    def invalidate(self) -> None:
        with self._lock:
            self.slot_map.invalidate()
