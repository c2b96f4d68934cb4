"""SLIDE slot redirection for one request/layer (reference ``slide.py``).

Host control plane: a token -> physical-slot map with pins, write guards,
copy-on-write promotion, completion-ordered publication, vacated-hole reuse
for decode and generation retirement.  The device copies it orders are done
by the caller's writer (``cacheslide_b200.paged`` uses the CUDA SLIDE
kernels).  Slot numbers are bit-exact with the reference: fresh sidecar
slots come lowest-first from ``allocation_floor`` (recycled ones first),
decode reuses the lowest eligible vacated hole.
"""

from __future__ import annotations

import threading
from collections import Counter
from collections.abc import Callable, Iterable, Iterator, Mapping
from concurrent.futures import Future
from contextlib import contextmanager
from dataclasses import dataclass

from .errors import CacheCapacityError, StaleCompletionError


@dataclass(frozen=True)
class SlotWrite:
    start_slot: int
    slot_count: int
    payload: bytes


def coalesce_slot_writes(writes: Mapping[int, bytes]) -> list[SlotWrite]:
    """Merge records of consecutive slots into runs (slide.py:27-51)."""
    if not writes:
        return []
    sizes = {len(payload) for payload in writes.values()}
    if len(sizes) != 1 or 0 in sizes:
        raise ValueError("token records must have one positive byte size")
    for slot, data in writes.items():
        if type(slot) is not int or slot < 0 or not isinstance(data, bytes):
            raise ValueError("slots must be nonnegative integers and records bytes")
    runs: list[SlotWrite] = []
    ordered = sorted(writes)
    start = ordered[0]
    parts = [writes[start]]
    for prev, slot in zip(ordered, ordered[1:]):
        if slot == prev + 1:
            parts.append(writes[slot])
            continue
        runs.append(SlotWrite(start, len(parts), b"".join(parts)))
        start, parts = slot, [writes[slot]]
    runs.append(SlotWrite(start, len(parts), b"".join(parts)))
    return runs


class LayerSlotMap:
    """Thread-safe token -> slot map of one request and layer (slide.py:54-520).

    Counters: ``_pins`` (readers), ``_writes`` (reserved destinations that
    reject new readers), ``_inflight`` (slots that must not be reused or
    overwritten).  ``invalidate`` retires the map for good; late completions
    raise ``StaleCompletionError`` instead of publishing.
    """

    def __init__(
        self,
        initial_slots: Mapping[int, int],
        *,
        shared_slots: Iterable[int] = (),
        max_slots: int | None = None,
        allocation_floor: int = 0,
    ):
        mapping = dict(initial_slots)
        for token, slot in mapping.items():
            if type(token) is not int or token < 0 or type(slot) is not int or slot < 0:
                raise ValueError("tokens and slots must be nonnegative integers")
        shared = set(shared_slots)
        if not shared <= set(mapping.values()):
            raise ValueError("shared slots must be present in the initial mapping")
        if type(allocation_floor) is not int or allocation_floor < 0:
            raise ValueError("allocation_floor must be a nonnegative integer")
        next_slot = max(allocation_floor, max(mapping.values(), default=-1) + 1)
        if max_slots is not None and (
            type(max_slots) is not int or max_slots < 0 or max_slots < next_slot
        ):
            raise ValueError("max_slots is smaller than the initial arena")
        self._map = mapping
        self._shared = shared
        self.allocation_floor = allocation_floor
        self.max_slots = max_slots
        self._next_slot = next_slot
        self._mutex = threading.RLock()
        self._pins: Counter[int] = Counter()
        self._inflight: Counter[int] = Counter()
        self._writes: Counter[int] = Counter()
        self._pending_tokens: set[int] = set()
        self._vacated: set[int] = set()
        self._unused: set[int] = set()
        self._generation = 0
        self._closed = False

    # ------------------------------------------------------------ internals
    def _check_open(self) -> None:
        if self._closed:
            raise StaleCompletionError("layer slot map is retired")

    def _busy(self, slot: int) -> bool:
        return bool(self._pins[slot] or self._inflight[slot])

    def _fresh_slot(self) -> int:
        if self._unused:
            slot = min(self._unused)
            self._unused.discard(slot)
            return slot
        if self.max_slots is not None and self._next_slot >= self.max_slots:
            raise CacheCapacityError("sidecar slot arena is full")
        slot, self._next_slot = self._next_slot, self._next_slot + 1
        return slot

    def _lowest_hole(self, *, native_only: bool) -> int | None:
        live = set(self._map.values())
        holes = [
            s
            for s in self._vacated
            if s not in live
            and s not in self._shared
            and not self._busy(s)
            and (not native_only or s < self.allocation_floor)
        ]
        return min(holes) if holes else None

    # ------------------------------------------------------------- readers
    def snapshot(self) -> dict[int, int]:
        with self._mutex:
            self._check_open()
            return dict(self._map)

    def page_metadata(
        self, page_size: int, selected_tokens: Iterable[int]
    ) -> tuple[dict[str, int | bool], ...]:
        """Per physical page: mapped/selected counts and guard flags."""
        if type(page_size) is not int or page_size < 1:
            raise ValueError("page_size must be a positive integer")
        selected = set(selected_tokens)
        with self._mutex:
            self._check_open()
            if any(type(t) is not int for t in selected) or not selected <= set(self._map):
                raise ValueError("selected tokens must have current logical mappings")
            mapped = Counter(slot // page_size for slot in self._map.values())
            chosen = Counter(self._map[t] // page_size for t in selected)
            shared = {s // page_size for s in self._shared}
            pinned = {s // page_size for s, c in self._pins.items() if c}
            inflight = {s // page_size for s, c in self._inflight.items() if c}
            blocked = shared | pinned | inflight
            return tuple(
                {
                    "page_id": page,
                    "mapped_tokens": mapped[page],
                    "selected_count": chosen[page],
                    "dirty": chosen[page] > 0,
                    "shared": page in shared,
                    "pinned": page in pinned,
                    "inflight": page in inflight,
                    "spill_eligible": page not in blocked,
                }
                for page in sorted(mapped)
            )

    @contextmanager
    def pin_slots(self, slots: Iterable[int]) -> Iterator[None]:
        wanted = set(slots)
        with self._mutex:
            self._check_open()
            if not wanted <= set(self._map.values()):
                raise ValueError("only currently mapped slots can be pinned")
            if any(self._writes[s] for s in wanted):
                raise RuntimeError("physical slots are being written")
            self._pins.update(wanted)
        try:
            yield
        finally:
            with self._mutex:
                self._pins.subtract(wanted)

    @contextmanager
    def pinned_mapping(self, tokens: Iterable[int]) -> Iterator[dict[int, int]]:
        """Atomically snapshot and pin the mappings of ``tokens``."""
        tokens = tuple(tokens)
        with self._mutex:
            self._check_open()
            if any(type(t) is not int or t < 0 for t in tokens):
                raise ValueError("tokens must be nonnegative integer positions")
            view = {t: self._map[t] for t in tokens}
            slots = set(view.values())
            if any(self._writes[s] for s in slots):
                raise RuntimeError("physical slots are being written")
            self._pins.update(slots)
        try:
            yield view
        finally:
            with self._mutex:
                self._pins.subtract(slots)

    # ------------------------------------------------------------- writers
    @contextmanager
    def write_guard(
        self, slots: Iterable[int], *, optional_slots: Iterable[int] = ()
    ) -> Iterator[frozenset[int]]:
        """Reserve physical writes; optional slots are skipped when guarded."""
        required_list, optional_list = tuple(slots), tuple(optional_slots)
        if any(type(s) is not int or s < 0 for s in required_list + optional_list):
            raise ValueError("write slots must be nonnegative integers")
        required = set(required_list)
        with self._mutex:
            self._check_open()
            if required & self._shared:
                raise ValueError("required write slots cannot be shared")
            if any(self._busy(s) for s in required):
                raise RuntimeError("required write slots are pinned or in-flight")
            usable = frozenset(
                s for s in set(optional_list) if s not in self._shared and not self._busy(s)
            )
            held = required | usable
            generation = self._generation
            self._writes.update(held)
            self._inflight.update(held)
        try:
            yield usable
            with self._mutex:
                if self._closed or generation != self._generation:
                    raise StaleCompletionError("write completed for a retired layer")
        finally:
            with self._mutex:
                self._writes.subtract(held)
                self._inflight.subtract(held)

    def promote_selected(
        self,
        updates: Mapping[int, bytes],
        writer: Callable[[list[SlotWrite]], Future | None],
        *,
        load_future: Future | None = None,
        allow_inplace: bool = False,
    ) -> Future[dict[int, int]]:
        """Write selected tokens, then atomically publish their new slots.

        Copy-on-write into fresh sidecar slots unless ``allow_inplace`` and the
        source is exclusive, idle and fully loaded (slide.py:243-372).
        """
        result: Future[dict[int, int]] = Future()
        result.set_running_or_notify_cancel()
        updates = dict(updates)
        coalesce_slot_writes({i: data for i, data in enumerate(updates.values())})
        with self._mutex:
            self._check_open()
            if not updates:
                result.set_result(dict(self._map))
                return result
            if not set(updates) <= set(self._map):
                raise KeyError("selected tokens must already have source slots")
            if self._pending_tokens & set(updates):
                raise RuntimeError("selected tokens already have an in-flight write")
            loading = load_future is not None and not load_future.done()
            if load_future is not None and not loading:
                load_future.result()
            generation = self._generation
            source = {t: self._map[t] for t in updates}
            uses = Counter(self._map.values())
            target: dict[int, int] = {}
            fresh: set[int] = set()
            try:
                for token, old in source.items():
                    copy = (
                        not allow_inplace
                        or loading
                        or old in self._shared
                        or self._busy(old)
                        or uses[old] > 1
                    )
                    dest = self._fresh_slot() if copy else old
                    target[token] = dest
                    if dest != old:
                        fresh.add(dest)
            except BaseException:
                self._unused.update(fresh)
                raise
            self._pending_tokens.update(updates)
            held = set(source.values()) | set(target.values())
            self._inflight.update(held)
            writing = set(target.values())
            self._writes.update(writing)
            if loading:
                sources = set(source.values())
                self._inflight.update(sources)

                def release_sources(_: Future) -> None:
                    with self._mutex:
                        self._inflight.subtract(sources)

                load_future.add_done_callback(release_sources)

        runs = coalesce_slot_writes({target[t]: data for t, data in updates.items()})

        def finish(done: Future | None = None, failure: BaseException | None = None) -> None:
            error: BaseException | None = None
            published = None
            try:
                if failure is not None:
                    raise failure
                if done is not None:
                    done.result()
                with self._mutex:
                    if self._closed or generation != self._generation:
                        raise StaleCompletionError(
                            "selected write completed for a retired layer"
                        )
                    if any(self._map[t] != s for t, s in source.items()):
                        raise StaleCompletionError("source mapping changed before publication")
                    self._map.update(target)
                    live = set(self._map.values())
                    for old in source.values():
                        if old not in live and old not in self._shared:
                            self._vacated.add(old)
                    published = dict(self._map)
            except BaseException as exc:
                with self._mutex:
                    self._unused.update(fresh)
                error = exc
            finally:
                with self._mutex:
                    self._writes.subtract(writing)
                    self._inflight.subtract(held)
                    self._pending_tokens.difference_update(updates)
            if error is not None:
                result.set_exception(error)
            else:
                result.set_result(published)

        try:
            written = writer(runs)
            if written is None:
                finish()
            elif isinstance(written, Future):
                written.add_done_callback(finish)
            else:
                raise TypeError("writer must return a concurrent Future or None")
        except BaseException as exc:
            finish(failure=exc)
        return result

    def allocate_decode(self, token: int) -> int:
        """Map a new decode token to the lowest idle hole, else a fresh slot."""
        with self._mutex:
            self._check_open()
            self._check_new_token(token)
            slot = self._lowest_hole(native_only=False)
            if slot is not None:
                self._vacated.discard(slot)
            else:
                slot = self._fresh_slot()
            self._map[token] = slot
            return slot

    def _check_new_token(self, token: int) -> None:
        if (
            type(token) is not int
            or token < 0
            or token in self._map
            or token in self._pending_tokens
        ):
            raise ValueError("decode token must be a new nonnegative position")

    def _decode_destination(self, token: int, physical_slot: int, *, reuse_vacated: bool) -> int:
        self._check_open()
        self._check_new_token(token)
        if type(physical_slot) is not int or not 0 <= physical_slot < self.allocation_floor:
            raise ValueError("native decode slot must be below allocation_floor")
        if (
            physical_slot in self._map.values()
            or physical_slot in self._shared
            or self._busy(physical_slot)
        ):
            raise CacheCapacityError("native decode slot is valid or guarded")
        if reuse_vacated:
            hole = self._lowest_hole(native_only=True)
            if hole is not None:
                return hole
        return physical_slot

    def bind_decode(self, token: int, physical_slot: int, *, reuse_vacated: bool = False) -> int:
        """Bind a caller-owned native slot (or the lowest native hole)."""
        with self._mutex:
            slot = self._decode_destination(token, physical_slot, reuse_vacated=reuse_vacated)
            self._vacated.discard(slot)
            self._map[token] = slot
            return slot

    @contextmanager
    def decode_write_guard(
        self, token: int, physical_slot: int, *, reuse_vacated: bool = False
    ) -> Iterator[int]:
        """Reserve decode + mirror destinations; publish after the body."""
        with self._mutex:
            slot = self._decode_destination(token, physical_slot, reuse_vacated=reuse_vacated)
            held = {slot, physical_slot}
            generation = self._generation
            self._vacated.discard(slot)
            self._pending_tokens.add(token)
            self._writes.update(held)
            self._inflight.update(held)
        try:
            yield slot
            with self._mutex:
                if self._closed or generation != self._generation:
                    raise StaleCompletionError("decode write completed for a retired layer")
                self._map[token] = slot
        except BaseException:
            with self._mutex:
                if not self._closed:
                    self.invalidate()
            raise
        finally:
            with self._mutex:
                self._writes.subtract(held)
                self._inflight.subtract(held)
                self._pending_tokens.discard(token)

    def invalidate(self) -> None:
        with self._mutex:
            self._generation += 1
            self._closed = True

    def stats(self) -> dict[str, int]:
        with self._mutex:
            return {
                "mapped_tokens": len(self._map),
                "vacated_slots": len(self._vacated),
                "shared_slots": len(self._shared),
                "pinned_slots": sum(1 for c in self._pins.values() if c > 0),
                "inflight_slots": sum(1 for c in self._inflight.values() if c > 0),
                "generation": self._generation,
            }
