"""Seeded random operation traces over a ``LayerSlotMap`` (test helper).

``drive(LayerSlotMap, seed)`` runs one deterministic sequence of slot-map
operations -- promotions with immediate, deferred and failing writers and
pending loads, decode allocation and native binding (plain and through the
write guard, with failures), write guards and pins held across other
operations, page metadata, statistics, retirement -- and returns what every
step returned or raised, as plain strings.  The same driver runs the
reference's slot map (``tests/golden/make_golden.py`` records the outcomes in
``tests/golden/slot_trace.json``) and this package's (``tests/test_slot_map.py``
replays the seeds and compares step by step), so slot numbers, published
maps, guard decisions and exception types/messages must agree exactly.
"""

from __future__ import annotations

import random
from concurrent.futures import Future


def _outcome(fn):
    try:
        return "ok " + repr(fn())
    except BaseException as exc:  # noqa: BLE001 - the trace records every failure
        return f"raise {type(exc).__name__}: {exc}"


def drive(LayerSlotMap, seed: int, steps: int = 120) -> list[str]:
    rng = random.Random(seed)
    n_tokens = rng.randint(3, 12)
    floor = rng.choice([0, 0, n_tokens, n_tokens + 4])
    native = list(range(n_tokens + 6))
    rng.shuffle(native)
    base = floor if floor else 0
    initial = {t: base + native[t] if floor == 0 else native[t] % max(floor, 1)
               for t in range(n_tokens)}
    if rng.random() < 0.3 and n_tokens > 2:  # two tokens sharing one slot
        initial[1] = initial[0]
    slots = sorted(set(initial.values()))
    shared = set(rng.sample(slots, k=min(len(slots), rng.randint(0, 2))))
    hi = max(max(initial.values()) + 1, floor)
    max_slots = rng.choice([None, hi + rng.randint(0, 6)])
    log: list[str] = []
    try:
        m = LayerSlotMap(dict(initial), shared_slots=shared, max_slots=max_slots,
                         allocation_floor=floor)
    except BaseException as exc:  # noqa: BLE001
        return [f"ctor raise {type(exc).__name__}: {exc}"]
    log.append(f"ctor {sorted(initial.items())} shared={sorted(shared)} "
               f"max={max_slots} floor={floor}")
    held = []          # open context managers
    writes = []        # (writer future, promotion future) pending
    loads = []         # pending load futures
    promotions = []    # promotion futures, read at the end
    next_token = n_tokens
    record = bytes([seed % 251 + 1]) * 4

    for step in range(steps):
        op = rng.choice(["promote", "promote", "promote", "decode", "bind", "guard_decode",
                         "write_guard", "pin", "pinned", "release", "release", "finish",
                         "finish", "load_done", "meta", "stats", "snapshot", "retire"])
        tokens = sorted(initial) + list(range(n_tokens, next_token))
        if op == "promote":
            chosen = rng.sample(tokens, k=min(len(tokens), rng.randint(0, 3)))
            if rng.random() < 0.1:
                chosen.append(10_000)  # unmapped token
            mode = rng.choice(["now", "later", "fail_now", "bad_type"])
            load = None
            if rng.random() < 0.4:
                load = Future()
                if rng.random() < 0.5:
                    load.set_result(None)
                else:
                    loads.append(load)
            inplace = rng.random() < 0.5
            runs_seen = []

            def writer(runs, mode=mode, runs_seen=runs_seen):
                runs_seen.append([(r.start_slot, r.slot_count, len(r.payload)) for r in runs])
                if mode == "now":
                    return None
                if mode == "fail_now":
                    raise OSError("writer failed")
                if mode == "bad_type":
                    return 7
                fut = Future()
                writes.append(fut)
                return fut

            def go():
                fut = m.promote_selected({t: record for t in chosen}, writer,
                                         load_future=load, allow_inplace=inplace)
                promotions.append(fut)
                return (fut.done(), runs_seen)

            log.append(f"{step} promote {chosen} {mode} inplace={inplace} "
                       f"load={'none' if load is None else load.done()}: {_outcome(go)}")
        elif op == "decode":
            t = next_token if rng.random() < 0.9 else rng.choice(tokens)
            res = _outcome(lambda: m.allocate_decode(t))
            if t == next_token and res.startswith("ok"):
                next_token += 1
            log.append(f"{step} decode {t}: {res}")
        elif op in ("bind", "guard_decode"):
            t = next_token
            phys = rng.randint(0, max(floor, 1) + 1)
            reuse = rng.random() < 0.6
            if op == "bind":
                res = _outcome(lambda: m.bind_decode(t, phys, reuse_vacated=reuse))
            else:
                fail = rng.random() < 0.15

                def guarded():
                    with m.decode_write_guard(t, phys, reuse_vacated=reuse) as chosen_slot:
                        if fail:
                            raise OSError("copy failed")
                        return chosen_slot

                res = _outcome(guarded)
            if res.startswith("ok"):
                next_token += 1
            log.append(f"{step} {op} {t} {phys} reuse={reuse}: {res}")
        elif op == "write_guard":
            pool = sorted(set(initial.values())) + list(range(hi, hi + 4))
            req = rng.sample(pool, k=rng.randint(0, 2))
            opt = rng.sample(pool, k=rng.randint(0, 2))
            cm = m.write_guard(req, optional_slots=opt)
            res = _outcome(lambda: sorted(cm.__enter__()))
            if res.startswith("ok"):
                held.append(cm)
            log.append(f"{step} write_guard {req} {opt}: {res}")
        elif op in ("pin", "pinned"):
            if op == "pin":
                pool = sorted(set(initial.values())) + [hi + 1]
                cm = m.pin_slots(rng.sample(pool, k=rng.randint(0, 2)))
                res = _outcome(lambda: cm.__enter__())
            else:
                cm = m.pinned_mapping(rng.sample(tokens + [9_999], k=rng.randint(0, 2)))
                res = _outcome(lambda: sorted(cm.__enter__().items()))
            if res.startswith("ok"):
                held.append(cm)
            log.append(f"{step} {op}: {res}")
        elif op == "release" and held:
            cm = held.pop(rng.randrange(len(held)))
            log.append(f"{step} release: {_outcome(lambda: cm.__exit__(None, None, None))}")
        elif op == "finish" and writes:
            fut = writes.pop(rng.randrange(len(writes)))
            if rng.random() < 0.2:
                fut.set_exception(OSError("rolled back"))
            else:
                fut.set_result(None)
            log.append(f"{step} finish: {_outcome(lambda: m.stats())}")
        elif op == "load_done" and loads:
            fut = loads.pop(rng.randrange(len(loads)))
            fut.set_result(None)
            log.append(f"{step} load_done: {_outcome(lambda: m.stats())}")
        elif op == "meta":
            ps = rng.choice([1, 2, 4, 16])
            sel = rng.sample(tokens, k=min(len(tokens), rng.randint(0, 3)))
            log.append(f"{step} meta {ps} {sel}: {_outcome(lambda: m.page_metadata(ps, sel))}")
        elif op == "stats":
            log.append(f"{step} stats: {_outcome(lambda: m.stats())}")
        elif op == "snapshot":
            log.append(f"{step} snapshot: {_outcome(lambda: sorted(m.snapshot().items()))}")
        elif op == "retire" and rng.random() < 0.05:
            m.invalidate()
            log.append(f"{step} retire")
    for fut in writes:
        fut.set_result(None)
    for fut in loads:
        fut.set_result(None)
    while held:
        cm = held.pop()
        log.append(f"end release: {_outcome(lambda: cm.__exit__(None, None, None))}")
    for i, fut in enumerate(promotions):
        log.append(f"promotion {i}: {_outcome(lambda: sorted(fut.result().items()))}")
    log.append(f"final stats: {_outcome(lambda: m.stats())}")
    log.append(f"final snapshot: {_outcome(lambda: sorted(m.snapshot().items()))}")
    return log
