"""SLIDE slot redirection for one request and one layer (host control plane).

Public contract (``src/cacheslide_vllm/slide.py:21-520``): ``SlotWrite``,
``coalesce_slot_writes`` and ``LayerSlotMap`` with the same methods, slot
numbers, exceptions and messages, so slot tables are bit-exact with the
reference and callers need no edits.  The bookkeeping is this module's own:

* ``_Book`` keeps one record per physical slot with four counters -- how many
  tokens map to it (``owners``), readers holding it (``pins``), writes
  reserved on it (``writes``) and operations that must not see it reused
  (``inflight``) -- so every guard test is O(1) instead of a scan of the map.
* ``_Sidecar`` hands out fresh sidecar slots: the lowest recycled slot (one
  given back by a failed promotion) from a min-heap, else the next never-used
  slot from ``allocation_floor`` upward, up to ``max_slots``.
* ``_Holes`` holds vacated slots (a promoted token's old slot once nothing
  maps to it) in a min-heap with lazy deletion; decode takes the lowest one
  that is idle at that moment.

Device copies are not done here: the caller's writer receives coalesced runs
and returns a ``Future`` that completes when its copies have (``paged.py``
uses the CUDA SLIDE kernels and a CUDA event).
"""

from __future__ import annotations

import heapq
import threading
from collections import defaultdict
from collections.abc import Callable, Iterable, Iterator, Mapping
from concurrent.futures import Future
from contextlib import contextmanager
from dataclasses import dataclass

from .errors import CacheCapacityError, StaleCompletionError


@dataclass(frozen=True)
class SlotWrite:
    """``slot_count`` equal-sized records written from ``start_slot`` on."""

    start_slot: int
    slot_count: int
    payload: bytes


def coalesce_slot_writes(writes: Mapping[int, bytes]) -> list[SlotWrite]:
    """Group records of consecutive slots into one write each (slide.py:27-51).

    Slots of one run share ``slot - rank`` in sorted order, which is the key
    the runs are cut on."""
    if not writes:
        return []
    size = {len(record) for record in writes.values()}
    if len(size) != 1 or 0 in size:
        raise ValueError("token records must have one positive byte size")
    for slot, record in writes.items():
        if type(slot) is not int or slot < 0 or not isinstance(record, bytes):
            raise ValueError("slots must be nonnegative integers and records bytes")
    ordered = sorted(writes)
    runs: list[SlotWrite] = []
    first = 0
    for rank in range(1, len(ordered) + 1):
        if rank == len(ordered) or ordered[rank] - rank != ordered[first] - first:
            chunk = ordered[first:rank]
            runs.append(SlotWrite(chunk[0], len(chunk), b"".join(writes[s] for s in chunk)))
            first = rank
    return runs


class _Record:
    __slots__ = ("owners", "pins", "writes", "inflight")

    def __init__(self) -> None:
        self.owners = self.pins = self.writes = self.inflight = 0


class _Book:
    """Per-slot counters.  ``busy`` = pinned or in flight: such a slot may be
    neither overwritten in place nor handed out again."""

    def __init__(self) -> None:
        self._rec: dict[int, _Record] = defaultdict(_Record)

    def get(self, slot: int) -> _Record:
        return self._rec[slot]

    def busy(self, slot: int) -> bool:
        r = self._rec.get(slot)
        return r is not None and (r.pins != 0 or r.inflight != 0)

    def owned(self, slot: int) -> bool:
        r = self._rec.get(slot)
        return r is not None and r.owners != 0

    def writing(self, slot: int) -> bool:
        r = self._rec.get(slot)
        return r is not None and r.writes != 0

    def add(self, field: str, slots: Iterable[int], delta: int) -> None:
        for s in slots:
            r = self._rec[s]
            setattr(r, field, getattr(r, field) + delta)

    def slots_with(self, field: str) -> list[int]:
        return [s for s, r in self._rec.items() if getattr(r, field) != 0]

    def count_with(self, field: str) -> int:
        return sum(1 for r in self._rec.values() if getattr(r, field) > 0)


class _Sidecar:
    """Fresh-slot source: recycled slots lowest first, then never-used ones."""

    def __init__(self, first: int, limit: int | None) -> None:
        self.next = first
        self.limit = limit
        self._heap: list[int] = []
        self._members: set[int] = set()

    def take(self) -> int:
        if self._heap:
            slot = heapq.heappop(self._heap)
            self._members.discard(slot)
            return slot
        if self.limit is not None and self.next >= self.limit:
            raise CacheCapacityError("sidecar slot arena is full")
        self.next += 1
        return self.next - 1

    def give_back(self, slots: Iterable[int]) -> None:
        for slot in slots:
            if slot not in self._members:
                self._members.add(slot)
                heapq.heappush(self._heap, slot)


class _Holes:
    """Vacated slots; ``lowest`` returns the lowest one passing ``usable``."""

    def __init__(self) -> None:
        self._heap: list[int] = []
        self.members: set[int] = set()

    def add(self, slot: int) -> None:
        if slot not in self.members:
            self.members.add(slot)
            heapq.heappush(self._heap, slot)

    def discard(self, slot: int) -> None:
        self.members.discard(slot)  # its heap entry is dropped when reached

    def lowest(self, usable: Callable[[int], bool], below: int | None = None) -> int | None:
        skipped: list[int] = []
        found = None
        while self._heap:
            slot = self._heap[0]
            if slot not in self.members:
                heapq.heappop(self._heap)
                continue
            if below is not None and slot >= below:
                break  # every later entry is larger still
            if usable(slot):
                found = slot
                break
            skipped.append(heapq.heappop(self._heap))
        for slot in skipped:
            heapq.heappush(self._heap, slot)
        return found


class LayerSlotMap:
    """Thread-safe token -> physical slot map of one request and layer.

    Fresh slots come from the caller's sidecar arena (``allocation_floor`` up
    to ``max_slots``); slots below the floor are the caller's native slots.
    Promotions publish their new mappings only when the writer's copies have
    completed; a promoted token's old slot becomes a hole for decode once no
    token maps to it.  ``invalidate`` retires the map for good: later calls
    and late completions raise ``StaleCompletionError``.
    """

    def __init__(
        self,
        initial_slots: Mapping[int, int],
        *,
        shared_slots: Iterable[int] = (),
        max_slots: int | None = None,
        allocation_floor: int = 0,
    ):
        table = dict(initial_slots)
        for token, slot in table.items():
            if type(token) is not int or token < 0 or type(slot) is not int or slot < 0:
                raise ValueError("tokens and slots must be nonnegative integers")
        book = _Book()
        for slot in table.values():
            book.get(slot).owners += 1
        shared = set(shared_slots)
        if any(not book.owned(s) for s in shared):
            raise ValueError("shared slots must be present in the initial mapping")
        if type(allocation_floor) is not int or allocation_floor < 0:
            raise ValueError("allocation_floor must be a nonnegative integer")
        first_free = max([allocation_floor] + [s + 1 for s in table.values()])
        if max_slots is not None and (
            type(max_slots) is not int or max_slots < 0 or max_slots < first_free
        ):
            raise ValueError("max_slots is smaller than the initial arena")
        self.allocation_floor = allocation_floor
        self.max_slots = max_slots
        self._table = table
        self._book = book
        self._shared = shared
        self._sidecar = _Sidecar(first_free, max_slots)
        self._holes = _Holes()
        self._pending: set[int] = set()  # tokens with a write not yet published
        self._lock = threading.RLock()
        self._epoch = 0
        self._retired = False

    # -------------------------------------------------------------- helpers
    def _live(self) -> None:
        if self._retired:
            raise StaleCompletionError("layer slot map is retired")

    def _idle_hole(self, slot: int) -> bool:
        return (not self._book.owned(slot) and slot not in self._shared
                and not self._book.busy(slot))

    def _remap(self, token: int, slot: int) -> None:
        old = self._table.get(token)
        if old is not None:
            self._book.get(old).owners -= 1
        self._table[token] = slot
        self._book.get(slot).owners += 1

    def _check_new_token(self, token: int) -> None:
        if (type(token) is not int or token < 0 or token in self._table
                or token in self._pending):
            raise ValueError("decode token must be a new nonnegative position")

    # -------------------------------------------------------------- readers
    def snapshot(self) -> dict[int, int]:
        with self._lock:
            self._live()
            return dict(self._table)

    def page_metadata(
        self, page_size: int, selected_tokens: Iterable[int]
    ) -> tuple[dict[str, int | bool], ...]:
        """Per physical page holding mapped tokens: token and selected-token
        counts and the guards that keep it from being spilled
        (slide.py:119-156).  ``dirty`` = holds a selected token."""
        if type(page_size) is not int or page_size < 1:
            raise ValueError("page_size must be a positive integer")
        chosen = set(selected_tokens)
        with self._lock:
            self._live()
            if any(type(t) is not int for t in chosen) or any(
                    t not in self._table for t in chosen):
                raise ValueError("selected tokens must have current logical mappings")
            tokens: dict[int, int] = defaultdict(int)
            for slot in self._book.slots_with("owners"):
                tokens[slot // page_size] += self._book.get(slot).owners
            picked: dict[int, int] = defaultdict(int)
            for t in chosen:
                picked[self._table[t] // page_size] += 1
            guard = {name: {s // page_size for s in self._book.slots_with(field)}
                     for name, field in (("pinned", "pins"), ("inflight", "inflight"))}
            guard["shared"] = {s // page_size for s in self._shared}
            pages = []
            for page in sorted(tokens):
                flags = {name: page in members for name, members in guard.items()}
                pages.append({
                    "page_id": page,
                    "mapped_tokens": tokens[page],
                    "selected_count": picked.get(page, 0),
                    "dirty": picked.get(page, 0) > 0,
                    "shared": flags["shared"],
                    "pinned": flags["pinned"],
                    "inflight": flags["inflight"],
                    "spill_eligible": not any(flags.values()),
                })
            return tuple(pages)

    def _pin(self, slots: set[int]) -> None:
        if any(self._book.writing(s) for s in slots):
            raise RuntimeError("physical slots are being written")
        self._book.add("pins", slots, +1)

    def _unpin(self, slots: set[int]) -> None:
        with self._lock:
            self._book.add("pins", slots, -1)

    @contextmanager
    def pin_slots(self, slots: Iterable[int]) -> Iterator[None]:
        """Hold mapped slots against writes and reuse for the body."""
        held = set(slots)
        with self._lock:
            self._live()
            if any(not self._book.owned(s) for s in held):
                raise ValueError("only currently mapped slots can be pinned")
            self._pin(held)
        try:
            yield
        finally:
            self._unpin(held)

    @contextmanager
    def pinned_mapping(self, tokens: Iterable[int]) -> Iterator[dict[int, int]]:
        """The current slots of ``tokens``, pinned for the body (a gather)."""
        tokens = tuple(tokens)
        with self._lock:
            self._live()
            if any(type(t) is not int or t < 0 for t in tokens):
                raise ValueError("tokens must be nonnegative integer positions")
            view = {t: self._table[t] for t in tokens}
            held = set(view.values())
            self._pin(held)
        try:
            yield view
        finally:
            self._unpin(held)

    # -------------------------------------------------------------- writers
    def _reserve(self, slots: set[int]) -> None:
        self._book.add("writes", slots, +1)
        self._book.add("inflight", slots, +1)

    def _release(self, slots: set[int]) -> None:
        with self._lock:
            self._book.add("writes", slots, -1)
            self._book.add("inflight", slots, -1)

    @contextmanager
    def write_guard(
        self, slots: Iterable[int], *, optional_slots: Iterable[int] = ()
    ) -> Iterator[frozenset[int]]:
        """Reserve physical writes for the body (slide.py:182-232).

        Required slots must be unshared and idle, or nothing is reserved;
        optional ones (canonical mirrors) are dropped when shared or busy and
        the body receives those that were kept.  Readers cannot pin a reserved
        slot.  Keep the guard until the device writes have completed."""
        required_seq, optional_seq = tuple(slots), tuple(optional_slots)
        for s in required_seq + optional_seq:
            if type(s) is not int or s < 0:
                raise ValueError("write slots must be nonnegative integers")
        required = set(required_seq)
        with self._lock:
            self._live()
            if not required.isdisjoint(self._shared):
                raise ValueError("required write slots cannot be shared")
            if any(self._book.busy(s) for s in required):
                raise RuntimeError("required write slots are pinned or in-flight")
            kept = frozenset(s for s in set(optional_seq)
                             if s not in self._shared and not self._book.busy(s))
            held = required | kept
            epoch = self._epoch
            self._reserve(held)
        try:
            yield kept
            with self._lock:
                if self._retired or epoch != self._epoch:
                    raise StaleCompletionError("write completed for a retired layer")
        finally:
            self._release(held)

    def _destinations(self, source: dict[int, int], in_place_ok: bool) -> dict[int, int]:
        """A destination per token: its own slot when it may be overwritten in
        place, else a fresh sidecar slot (all given back if the arena runs out)."""
        dest: dict[int, int] = {}
        taken: list[int] = []
        try:
            for token, old in source.items():
                rec = self._book.get(old)
                own = (in_place_ok and old not in self._shared and rec.pins == 0
                       and rec.inflight == 0 and rec.owners <= 1)
                if own:
                    dest[token] = old
                else:
                    dest[token] = self._sidecar.take()
                    taken.append(dest[token])
        except BaseException:
            self._sidecar.give_back(taken)
            raise
        return dest

    def promote_selected(
        self,
        updates: Mapping[int, bytes],
        writer: Callable[[list[SlotWrite]], Future | None],
        *,
        load_future: Future | None = None,
        allow_inplace: bool = False,
    ) -> Future[dict[int, int]]:
        """Write new records of selected tokens, then publish their slots.

        A token's record goes to a fresh sidecar slot (copy-on-write) unless
        ``allow_inplace`` and its slot is exclusive, unshared, idle and its
        load has finished (slide.py:243-372).  ``writer(runs)`` gets the
        coalesced writes and returns ``None`` (done) or a ``Future``; the
        returned future resolves to the published map, or to the write's
        error (the fresh slots are then given back)."""
        result: Future[dict[int, int]] = Future()
        result.set_running_or_notify_cancel()
        updates = dict(updates)
        # reject malformed records before any slot is taken
        coalesce_slot_writes(dict(enumerate(updates.values())))
        with self._lock:
            self._live()
            if not updates:
                result.set_result(dict(self._table))
                return result
            if any(t not in self._table for t in updates):
                raise KeyError("selected tokens must already have source slots")
            if not self._pending.isdisjoint(updates):
                raise RuntimeError("selected tokens already have an in-flight write")
            loading = load_future is not None and not load_future.done()
            if load_future is not None and not loading:
                load_future.result()  # a failed load never allows in-place writes
            epoch = self._epoch
            source = {t: self._table[t] for t in updates}
            dest = self._destinations(source, allow_inplace and not loading)
            fresh = [d for t, d in dest.items() if d != source[t]]
            self._pending.update(updates)
            targets = set(dest.values())
            guarded = set(source.values()) | targets
            self._book.add("inflight", guarded, +1)
            self._book.add("writes", targets, +1)
            if loading:
                # sources still being loaded stay guarded until the load ends
                loading_slots = set(source.values())
                self._book.add("inflight", loading_slots, +1)
                load_future.add_done_callback(
                    lambda _f: self._with_lock(self._book.add, "inflight", loading_slots, -1))

        runs = coalesce_slot_writes({dest[t]: rec for t, rec in updates.items()})

        def publish() -> dict[int, int]:
            with self._lock:
                if self._retired or epoch != self._epoch:
                    raise StaleCompletionError("selected write completed for a retired layer")
                if any(self._table[t] != s for t, s in source.items()):
                    raise StaleCompletionError("source mapping changed before publication")
                for t, s in dest.items():
                    self._remap(t, s)
                for old in source.values():
                    if not self._book.owned(old) and old not in self._shared:
                        self._holes.add(old)
                return dict(self._table)

        def finish(done: Future | None = None, failure: BaseException | None = None) -> None:
            outcome: dict[int, int] | BaseException
            try:
                if failure is not None:
                    raise failure
                if done is not None:
                    done.result()
                outcome = publish()
            except BaseException as exc:
                with self._lock:
                    self._sidecar.give_back(fresh)
                outcome = exc
            finally:
                with self._lock:
                    self._book.add("writes", targets, -1)
                    self._book.add("inflight", guarded, -1)
                    self._pending.difference_update(updates)
            if isinstance(outcome, BaseException):
                result.set_exception(outcome)
            else:
                result.set_result(outcome)

        try:
            pending = writer(runs)
            if pending is None:
                finish()
            elif isinstance(pending, Future):
                pending.add_done_callback(finish)
            else:
                raise TypeError("writer must return a concurrent Future or None")
        except BaseException as exc:
            finish(failure=exc)
        return result

    def _with_lock(self, fn, *args) -> None:
        with self._lock:
            fn(*args)

    # --------------------------------------------------------------- decode
    def allocate_decode(self, token: int) -> int:
        """Map a new decode token to the lowest idle hole, else a fresh slot."""
        with self._lock:
            self._live()
            self._check_new_token(token)
            slot = self._holes.lowest(self._idle_hole)
            if slot is None:
                slot = self._sidecar.take()
            else:
                self._holes.discard(slot)
            self._remap(token, slot)
            return slot

    def _native_destination(self, token: int, physical_slot: int, reuse_vacated: bool) -> int:
        self._live()
        self._check_new_token(token)
        if type(physical_slot) is not int or not 0 <= physical_slot < self.allocation_floor:
            raise ValueError("native decode slot must be below allocation_floor")
        if (self._book.owned(physical_slot) or physical_slot in self._shared
                or self._book.busy(physical_slot)):
            raise CacheCapacityError("native decode slot is valid or guarded")
        if reuse_vacated:
            hole = self._holes.lowest(self._idle_hole, below=self.allocation_floor)
            if hole is not None:
                return hole
        return physical_slot

    def bind_decode(self, token: int, physical_slot: int, *, reuse_vacated: bool = False) -> int:
        """Map a new decode token to a caller-owned native slot below the floor,
        or, with ``reuse_vacated``, to the lowest idle native hole (the given
        slot is still checked, so the caller can mirror its write there)."""
        with self._lock:
            slot = self._native_destination(token, physical_slot, reuse_vacated)
            self._holes.discard(slot)
            self._remap(token, slot)
            return slot

    @contextmanager
    def decode_write_guard(
        self, token: int, physical_slot: int, *, reuse_vacated: bool = False
    ) -> Iterator[int]:
        """``bind_decode`` whose mapping is published only after the body (the
        device write) succeeds; both destinations are reserved meanwhile.  A
        failure retires the whole map (the write may be partial)."""
        with self._lock:
            slot = self._native_destination(token, physical_slot, reuse_vacated)
            held = {slot, physical_slot}
            epoch = self._epoch
            self._holes.discard(slot)
            self._pending.add(token)
            self._reserve(held)
        try:
            yield slot
            with self._lock:
                if self._retired or epoch != self._epoch:
                    raise StaleCompletionError("decode write completed for a retired layer")
                self._remap(token, slot)
        except BaseException:
            with self._lock:
                if not self._retired:
                    self.invalidate()
            raise
        finally:
            self._release(held)
            with self._lock:
                self._pending.discard(token)

    # ------------------------------------------------------------ lifecycle
    def invalidate(self) -> None:
        with self._lock:
            self._epoch += 1
            self._retired = True

    def stats(self) -> dict[str, int]:
        with self._lock:
            return {
                "mapped_tokens": len(self._table),
                "vacated_slots": len(self._holes.members),
                "shared_slots": len(self._shared),
                "pinned_slots": self._book.count_with("pins"),
                "inflight_slots": self._book.count_with("inflight"),
                "generation": self._epoch,
            }
