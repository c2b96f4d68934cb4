"""SLIDE host control plane (LayerSlotMap) on CPU: exact slot numbers.

Scenarios restate the reference's tests/test_slide.py: coalescing,
copy-on-write while a load is pending, in-place promotion, guards, shared
slots, hole reuse for decode, retirement.  No device work is involved.
"""

from __future__ import annotations

from concurrent.futures import Future

import pytest

from cacheslide_b200.errors import CacheCapacityError, StaleCompletionError
from cacheslide_b200.slide import LayerSlotMap, SlotWrite, coalesce_slot_writes


def test_coalesce_adjacent_records():
    assert coalesce_slot_writes({4: b"dd", 2: b"bb", 1: b"aa"}) == [
        SlotWrite(1, 2, b"aabb"),
        SlotWrite(4, 1, b"dd"),
    ]
    with pytest.raises(ValueError):
        coalesce_slot_writes({0: b"a", 1: b"bb"})
    assert coalesce_slot_writes({}) == []


def test_pending_load_copy_on_write_and_reclaim_after_load():
    layer = LayerSlotMap({0: 0, 1: 1, 2: 2}, max_slots=6)
    loading, writing = Future(), Future()
    seen = []
    done = layer.promote_selected({1: b"new"}, lambda runs: seen.extend(runs) or writing,
                                  load_future=loading)
    assert seen == [SlotWrite(3, 1, b"new")]
    assert layer.snapshot() == {0: 0, 1: 1, 2: 2}
    assert layer.allocate_decode(3) == 4
    writing.set_result(None)
    assert done.result()[1] == 3
    assert layer.allocate_decode(4) == 5
    with pytest.raises(CacheCapacityError):
        layer.allocate_decode(5)
    loading.set_result(None)
    assert layer.allocate_decode(5) == 1


def test_inplace_promotion_when_loaded_and_exclusive():
    loaded = Future()
    loaded.set_result(None)
    layer = LayerSlotMap({0: 0, 1: 1}, max_slots=2)
    seen = []
    result = layer.promote_selected({1: b"x"}, lambda runs: seen.extend(runs),
                                    load_future=loaded, allow_inplace=True)
    assert result.result() == {0: 0, 1: 1}
    assert seen == [SlotWrite(1, 1, b"x")]
    assert layer.stats()["vacated_slots"] == 0


@pytest.mark.parametrize("outcome", ["success", "failure", "retired"])
def test_async_inplace_rejects_pins_and_writers(outcome):
    layer = LayerSlotMap({0: 0, 1: 1}, max_slots=2)
    written = Future()
    done = layer.promote_selected({0: b"new"}, lambda _: written, allow_inplace=True)
    assert not done.done()
    for pin in (layer.pin_slots([0]), layer.pinned_mapping([0])):
        with pytest.raises(RuntimeError, match="being written"):
            with pin:
                pass
    with pytest.raises(RuntimeError, match="in-flight"):
        with layer.write_guard([0]):
            pass
    if outcome == "retired":
        layer.invalidate()
    if outcome == "failure":
        written.set_exception(OSError("rolled back"))
        with pytest.raises(OSError, match="rolled back"):
            done.result()
    else:
        written.set_result(None)
        if outcome == "retired":
            with pytest.raises(StaleCompletionError):
                done.result()
        else:
            assert done.result() == {0: 0, 1: 1}
    assert layer.stats()["inflight_slots"] == 0


def test_guard_forces_independent_destination_and_shared_never_reclaimed():
    layer = LayerSlotMap({0: 0}, max_slots=2)
    written = Future()
    with layer.write_guard([0]):
        done = layer.promote_selected({0: b"new"}, lambda _: written, allow_inplace=True)
        written.set_result(None)
        assert done.result() == {0: 1}
        with pytest.raises(CacheCapacityError):
            layer.allocate_decode(1)
    assert layer.allocate_decode(1) == 0
    shared = LayerSlotMap({0: 0, 1: 1}, shared_slots={1}, max_slots=4)
    assert shared.promote_selected({1: b"x"}, lambda runs: None,
                                   allow_inplace=True).result()[1] == 2
    assert shared.allocate_decode(2) == 3
    with pytest.raises(CacheCapacityError):
        shared.allocate_decode(3)


def test_decode_binds_native_slot_or_lowest_native_hole():
    layer = LayerSlotMap({0: 0, 1: 1, 2: 2}, allocation_floor=8, max_slots=12)
    layer.promote_selected({1: b"a", 0: b"b"}, lambda runs: None).result()
    assert layer.snapshot() == {0: 9, 1: 8, 2: 2}
    with pytest.raises(ValueError, match="below allocation_floor"):
        layer.bind_decode(3, 8)
    with pytest.raises(CacheCapacityError, match="valid or guarded"):
        layer.bind_decode(3, 2)
    with layer.decode_write_guard(3, 5, reuse_vacated=True) as chosen:
        assert chosen == 0
    assert layer.bind_decode(4, 6, reuse_vacated=True) == 1
    assert layer.bind_decode(5, 7, reuse_vacated=True) == 7
    with pytest.raises(ValueError, match="new nonnegative"):
        layer.bind_decode(5, 4)


def test_failed_decode_write_retires_the_map():
    layer = LayerSlotMap({0: 0}, allocation_floor=4, max_slots=6)
    with pytest.raises(OSError):
        with layer.decode_write_guard(1, 1):
            raise OSError("copy failed")
    with pytest.raises(StaleCompletionError):
        layer.snapshot()


def test_page_metadata_counts_and_guards():
    layer = LayerSlotMap({0: 0, 1: 1, 2: 5, 3: 6}, shared_slots={6}, max_slots=10)
    meta = {p["page_id"]: p for p in layer.page_metadata(4, [0, 2])}
    assert meta[0]["selected_count"] == 1 and meta[1]["selected_count"] == 1
    assert meta[1]["shared"] and not meta[1]["spill_eligible"]
    with layer.pin_slots([0]):
        assert next(p for p in layer.page_metadata(4, []) if p["page_id"] == 0)["pinned"]


def test_random_traces_match_the_reference_slot_map():
    """Seeded random operation traces (tests/slot_trace.py) give exactly the
    reference LayerSlotMap's outcomes: every slot number, published map,
    guard decision, statistic and exception (tests/golden/slot_trace.json,
    recorded from the reference by tests/golden/make_golden.py)."""
    import hashlib
    import json
    from pathlib import Path

    import slot_trace

    golden = json.loads((Path(__file__).parent / "golden" / "slot_trace.json").read_text())
    assert golden["steps"] == 120
    bad = []
    for seed, want in golden["seeds"].items():
        lines = slot_trace.drive(LayerSlotMap, int(seed))
        got = hashlib.sha256("\n".join(lines).encode()).hexdigest()
        if len(lines) != want["lines"] or got != want["sha256"]:
            bad.append(int(seed))
    assert not bad, f"traces differ from the reference for seeds {bad[:10]}"


def test_errors_are_the_reference_classes_when_it_is_importable():
    """With the reference package on the path, the slot map raises the
    reference's own storage errors, so its runtime's fallbacks catch them
    unedited; without it, classes of the same names and bases are used."""
    import subprocess
    import sys
    from pathlib import Path

    from cacheslide_b200 import errors

    assert issubclass(errors.CacheCapacityError, RuntimeError)
    stub = Path(__file__).parent / "_stub_reference"
    code = (
        "import sys; sys.path.insert(0, %r)\n"
        "from cacheslide_vllm.storage import CacheCapacityError as Ref\n"
        "from cacheslide_b200 import errors\n"
        "from cacheslide_b200.slide import LayerSlotMap\n"
        "assert errors.SHARED_WITH_REFERENCE and errors.CacheCapacityError is Ref\n"
        "m = LayerSlotMap({0: 0}, max_slots=1)\n"
        "try:\n    m.allocate_decode(1)\nexcept Ref:\n    print('caught')\n"
    ) % str(stub)
    out = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                         cwd=str(Path(__file__).parents[1]))
    assert out.returncode == 0, out.stderr
    assert out.stdout.strip() == "caught"
