"""Generate golden vectors by running the reference CacheSlide implementation.

Run in a container that has the reference source checkout:

    python tests/golden/make_golden.py /path/to/CacheSlide/src

It imports ``cacheslide_vllm`` from that path, runs its own CoPE attention,
position policies, WCA state machine and paged arena on seeded inputs, and
writes small ``.npz`` fixtures next to this script.  The tests compare the
numpy oracle and the CUDA library against these files; the GPU box never needs
the reference itself.
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _np(t):
    return t.detach().cpu().clone().numpy()


def _bf16(t):
    return t.to(torch.bfloat16).to(torch.float32)


def cope_cases(ref):
    from cacheslide_vllm.attention import (
        CanonicalPositionPolicy,
        SelectedAssociationPolicy,
    )
    from cacheslide_vllm.contracts import RequestPlan
    from cacheslide_vllm.position import (
        CCPEPositionError,
        CCPEProfile,
        ChunkIdentity,
        CoPE,
        cope_attention,
    )

    out = {}
    g = torch.Generator().manual_seed(0)
    # -- plain CoPE, GQA, arbitrary sorted query rows, bf16-valued inputs ----
    nk, hq, hkv, d, npos = 96, 4, 2, 32, 16
    q = _bf16(torch.randn(nk, hq, d, generator=g))
    k = _bf16(torch.randn(nk, hkv, d, generator=g))
    v = _bf16(torch.randn(nk, hkv, d, generator=g))
    E = _bf16(torch.randn(d, npos, generator=g) * 0.5)
    rows = torch.sort(torch.randperm(nk, generator=g)[:40]).values
    cope = CoPE(d, npos)
    with torch.no_grad():
        cope.position_embeddings.copy_(E)
    o, p = cope_attention(
        q[rows], k, v, cope, rows, query_chunk_size=16, return_positions=True
    )
    out["plain"] = dict(q=_np(q[rows]), k=_np(k), v=_np(v), E=_np(E),
                        qpos=_np(rows), out=_np(o), positions=_np(p))
    # -- decode: one row at the last position -------------------------------
    last = torch.tensor([nk - 1])
    o = cope_attention(q[-1:], k, v, cope, last)
    out["decode"] = dict(q=_np(q[-1:]), k=_np(k), v=_np(v), E=_np(E),
                         qpos=_np(last), out=_np(o))
    # -- sparse key coordinates --------------------------------------------
    kpos = torch.sort(torch.randperm(3 * nk, generator=g)[:nk]).values
    qsel = kpos[rows]
    o = cope_attention(q[rows], k, v, cope, qsel, kpos, query_chunk_size=7)
    out["sparse_keys"] = dict(q=_np(q[rows]), k=_np(k), v=_np(v), E=_np(E),
                              qpos=_np(qsel), kpos=_np(kpos), out=_np(o))
    # -- WCA association visibility (applied after gates) --------------------
    fixed = tuple(int(i) for i in range(nk) if (i // 16) % 3 != 1)
    selected = torch.tensor([i for i in fixed if i % 5 == 0])
    assoc = SelectedAssociationPolicy(fixed, selected)
    o = cope_attention(q[rows], k, v, cope, rows, visibility_transform=assoc,
                       query_chunk_size=9)
    out["assoc"] = dict(q=_np(q[rows]), k=_np(k), v=_np(v), E=_np(E),
                        qpos=_np(rows), out=_np(o), fixed=np.array(fixed),
                        selected=_np(selected))
    # -- attention_mask (gates + attention) and visibility_mask --------------
    am = torch.rand(len(rows), nk, generator=g) > 0.2
    vm = torch.rand(hq, len(rows), nk, generator=g) > 0.3
    o = cope_attention(q[rows], k, v, cope, rows, attention_mask=am,
                       visibility_mask=vm, query_chunk_size=11)
    out["masks"] = dict(q=_np(q[rows]), k=_np(k), v=_np(v), E=_np(E),
                        qpos=_np(rows), out=_np(o), attention_mask=_np(am),
                        visibility_mask=_np(vm))

    # -- canonical CCPE table substitution (mixed and strict) ---------------
    def plan_for(layout):
        chunks, cursor, seen = [], 0, {"reuse": 0, "recompute": 0}
        for role, length in layout:
            name = ("u" if role == "reuse" else "d") + str(seen[role])
            seen[role] += 1
            chunks.append({"id": name, "role": role, "start": cursor,
                           "end": cursor + length})
            cursor += length
        ids = [(7 * j + 3) % 50 for j in range(cursor)]
        return RequestPlan.parse({"version": 1, "namespace": "golden",
                                  "task_id": "ccpe", "operation": "reuse",
                                  "chunks": chunks}, ids)

    calib_layout = [("reuse", 16), ("reuse", 16), ("reuse", 16)]
    calib_plan = plan_for(calib_layout)
    nfix = len(calib_plan.fixed_indices)
    qc = _bf16(torch.randn(nfix, hq, d, generator=g))
    kc = _bf16(torch.randn(nfix, hkv, d, generator=g))
    trace = cope.position_trace(qc, kc, torch.arange(nfix), checkpoint_id="ck")
    fixed_t = torch.tensor(calib_plan.fixed_indices)
    profile = CCPEProfile.calibrate(
        [trace.project(fixed_t, fixed_t)],
        [ChunkIdentity(*e) for e in calib_plan.fixed_layout],
        trained_profile_version="golden-v1",
    )
    live_layout = [("reuse", 16), ("recompute", 8), ("reuse", 16), ("reuse", 16),
                   ("recompute", 4)]
    live = plan_for(live_layout)
    # token ids of reused chunks must match the calibration layout's hashes
    ids = list(live.token_ids)
    src = list(calib_plan.token_ids)
    live_fixed = live.fixed_indices
    for o_i, pos in enumerate(live_fixed):
        ids[pos] = src[calib_plan.fixed_indices[o_i]]
    live = RequestPlan.parse(json.loads(live.to_json()), ids)
    n_live = len(ids)
    ql = _bf16(torch.randn(n_live, hq, d, generator=g))
    kl = _bf16(torch.randn(n_live, hkv, d, generator=g))
    vl = _bf16(torch.randn(n_live, hkv, d, generator=g))
    qrows = torch.arange(n_live)
    mixed = CanonicalPositionPolicy(live, profile, "ck", mode="mixed_bias_override")
    o, p = cope_attention(ql, kl, vl, cope, qrows, positions_transform=mixed,
                          query_chunk_size=13, return_positions=True)
    out["canonical_mixed"] = dict(
        q=_np(ql), k=_np(kl), v=_np(vl), E=_np(E), qpos=_np(qrows), out=_np(o),
        positions=_np(p), fixed=np.array(live_fixed),
        table=_np(profile.canonical_positions),
        table_query_positions=_np(profile.query_positions))
    strict = CanonicalPositionPolicy(live, profile, "ck", mode="strict_contextual")
    try:
        cope_attention(ql, kl, vl, cope, qrows, positions_transform=strict,
                       query_chunk_size=13)
        message = ""
    except CCPEPositionError as error:
        message = str(error)
    out["canonical_mixed"]["strict_error"] = np.array(message)
    # same layout as calibration: strict accepts (actual contextual path)
    qs = qc.clone()
    o = cope_attention(qs, kc, kc, cope, torch.arange(nfix),
                       positions_transform=CanonicalPositionPolicy(
                           calib_plan, profile, "ck"), query_chunk_size=8)
    out["canonical_strict_ok"] = dict(
        q=_np(qs), k=_np(kc), v=_np(kc), E=_np(E), qpos=np.arange(nfix),
        out=_np(o), fixed=np.array(calib_plan.fixed_indices),
        table=_np(profile.canonical_positions),
        table_query_positions=_np(profile.query_positions))
    # -- fixed positions: reference bias/softmax on externally given positions
    fpos = torch.rand(hq, len(rows), nk, generator=g) * (npos - 1)
    o = cope_attention(q[rows], k, v, cope, rows, fixed_positions=fpos)
    out["fixed_positions"] = dict(q=_np(q[rows]), k=_np(k), v=_np(v), E=_np(E),
                                  qpos=_np(rows), out=_np(o), positions=_np(fpos))
    return out


def wca_cases(ref):
    from cacheslide_vllm.wca import WCAConfig, WCAState, mean_head_cosine

    out = {}
    g = torch.Generator().manual_seed(1)
    n, hkv, d = 80, 2, 16
    reused = torch.ones(n, dtype=torch.bool)
    reused[32:44] = False
    mandatory = ~reused
    mandatory[n - 1] = True
    cached = _bf16(torch.randn(n, hkv, d, generator=g))
    fresh = _bf16(cached + 0.3 * torch.randn(n, hkv, d, generator=g))
    # plant exact ties to pin the stable index tie-break
    fresh[5], cached[5] = cached[9] + 1, cached[9]
    fresh[9] = cached[9] + 1
    fresh[~reused] = cached[~reused]
    cfg = WCAConfig(correction_fraction=0.15, gate_interval=2)
    state = WCAState.initialize(cached, fresh, reused, mandatory, cfg)
    rec = dict(cached=_np(cached), fresh=_np(fresh), reused=_np(reused),
               mandatory=_np(mandatory), budget=np.array(state.budget),
               deviation=_np(state.initial_deviation), alpha0=_np(state.alpha),
               active1=_np(state.active_indices))
    for layer in (2, 3, 4):
        ck = _bf16(torch.randn(n, hkv, d, generator=g))
        cv = _bf16(torch.randn(n, hkv, d, generator=g))
        rows = state.active_indices
        fk = _bf16(ck[rows] + 0.5 * torch.randn(len(rows), hkv, d, generator=g))
        fv = _bf16(cv[rows] + 0.5 * torch.randn(len(rows), hkv, d, generator=g))
        if layer == 4:
            fk[::2] = -ck[rows][::2]  # force some low cosines
        upd = state.update(layer, ck, cv, fk, fv)
        rec.update({
            f"L{layer}_ck": _np(ck), f"L{layer}_cv": _np(cv),
            f"L{layer}_fk": _np(fk), f"L{layer}_fv": _np(fv),
            f"L{layer}_indices": _np(upd.indices),
            f"L{layer}_fused_k": _np(upd.fused_k.to(torch.float32)),
            f"L{layer}_fused_v": _np(upd.fused_v.to(torch.float32)),
            f"L{layer}_alpha": _np(upd.alpha),
            f"L{layer}_removed": _np(upd.removed_indices),
            f"L{layer}_promoted": _np(upd.promoted_indices),
            f"L{layer}_next": _np(upd.next_indices),
        })
    out["sequence"] = rec
    a = _bf16(torch.randn(40, 4, 16, generator=g))
    b = _bf16(a + torch.randn(40, 4, 16, generator=g))
    b[3] = 0
    out["cosine"] = dict(a=_np(a), b=_np(b), cos=_np(mean_head_cosine(a, b)))
    return out


def paged_cases(ref):
    from concurrent.futures import Future

    from cacheslide_vllm.paged import NativePagedKV

    g = torch.Generator().manual_seed(2)
    out = {}
    # bf16 records on a shuffled block table; raw bits compared exactly
    nb, hkv, bs, d = 12, 2, 4, 8
    cache = torch.zeros(nb, hkv, bs, 2 * d, dtype=torch.bfloat16)
    table = [7, 2, 9, 0, 5]
    arena = NativePagedKV(cache, table, 18, 4, request_id="g", layer_index=1)
    key = torch.randn(18, hkv, d, generator=g).to(torch.bfloat16)
    value = torch.randn(18, hkv, d, generator=g).to(torch.bfloat16)
    arena.write_prefill(key, value)
    snap0 = arena.snapshot()
    loading = Future()
    sel = [3, 11, 6]
    m1 = arena.promote_selected(sel, key[sel] + 1, value[sel] - 1,
                                load_future=loading).result()
    loading.set_result(None)
    arena.write_prefill(key, value)
    upd = [3, 6, 11, 17]
    uk, uv = key[upd] * 2, value[upd] * 3
    arena.update_selected(upd, uk, uv)
    d1 = arena.decode(18, key[0] + 5, value[0] + 5)
    d2 = arena.decode(19, key[1] + 6, value[1] + 6)
    order = list(range(20))[::-1]
    gk, gv = arena.gather(order)
    out["arena"] = dict(
        table=np.array(table), key=_np(key.view(torch.int16)),
        value=_np(value.view(torch.int16)),
        snap0=np.array([snap0[t] for t in range(18)]),
        promoted=np.array([m1[t] for t in sel]), decode=np.array([d1, d2]),
        final_map=np.array([arena.snapshot()[t] for t in range(20)]),
        order=np.array(order), gathered_k=_np(gk.view(torch.int16)),
        gathered_v=_np(gv.view(torch.int16)),
        cache=_np(cache.view(torch.int16)),
        side_k=_np(arena._side_key.view(torch.int16)),
        side_v=_np(arena._side_value.view(torch.int16)),
        stats=np.array(json.dumps(arena.stats(), sort_keys=True)))
    return out


def profile_cases(ref):
    """A CCPE profile calibrated by the reference from three prompts that
    share their fixed chunks (the same Q/K rows) and differ in their dynamic
    tokens, and the reference's canonical-table attention
    (CanonicalPositionPolicy, mixed_bias_override) on each prompt: the
    fixtures of the compressed per-chunk form (cs_cope_chunk_offsets)."""
    from cacheslide_vllm.attention import CanonicalPositionPolicy
    from cacheslide_vllm.contracts import RequestPlan
    from cacheslide_vllm.position import CCPEProfile, ChunkIdentity, CoPE, cope_attention

    g = torch.Generator().manual_seed(7)
    hq, hkv, d, npos = 4, 2, 32, 16
    layout = [("reuse", 12), ("recompute", 5), ("reuse", 9), ("reuse", 10), ("recompute", 4)]
    chunks, cursor = [], 0
    for i, (role, length) in enumerate(layout):
        chunks.append({"id": f"c{i}", "role": role, "start": cursor, "end": cursor + length})
        cursor += length
    n = cursor
    ids = [(5 * j + 1) % 40 for j in range(n)]
    plan = RequestPlan.parse({"version": 1, "namespace": "golden", "task_id": "ccpe-compressed",
                              "operation": "reuse", "chunks": chunks}, ids)
    fixed = torch.tensor(plan.fixed_indices)
    E = _bf16(torch.randn(d, npos, generator=g) * 0.5)
    cope = CoPE(d, npos)
    with torch.no_grad():
        cope.position_embeddings.copy_(E)
    qf = _bf16(torch.randn(fixed.numel(), hq, d, generator=g))
    kf = _bf16(torch.randn(fixed.numel(), hkv, d, generator=g))
    vf = _bf16(torch.randn(fixed.numel(), hkv, d, generator=g))
    prompts, traces = [], []
    for _ in range(3):
        q = _bf16(torch.randn(n, hq, d, generator=g))
        k = _bf16(torch.randn(n, hkv, d, generator=g))
        v = _bf16(torch.randn(n, hkv, d, generator=g))
        q[fixed], k[fixed], v[fixed] = qf, kf, vf  # same fixed content
        prompts.append((q, k, v))
        trace = cope.position_trace(q, k, torch.arange(n), checkpoint_id="ck")
        traces.append(trace.project(fixed, fixed))
    profile = CCPEProfile.calibrate(traces, [ChunkIdentity(*e) for e in plan.fixed_layout],
                                    trained_profile_version="golden-v1")
    rep = [i for i, t in enumerate(traces)
           if torch.equal(t.positions, profile.canonical_positions)][0]
    out = {"meta": dict(fixed=_np(fixed),
                        chunk_lengths=np.array([e[2] for e in plan.fixed_layout]),
                        n=np.array(n), E=_np(E), representative=np.array(rep),
                        table=_np(profile.canonical_positions),
                        table_query_positions=_np(profile.query_positions))}
    policy = CanonicalPositionPolicy(plan, profile, "ck", mode="mixed_bias_override")
    for i, (q, k, v) in enumerate(prompts):
        o, p = cope_attention(q, k, v, cope, torch.arange(n), positions_transform=policy,
                              query_chunk_size=11, return_positions=True)
        out[f"prompt{i}"] = dict(q=_np(q), k=_np(k), v=_np(v), out=_np(o), positions=_np(p))
    return out


SLOT_TRACE_SEEDS = 400


def slot_traces(ref) -> dict:
    """The reference's LayerSlotMap driven through the seeded random traces of
    ``tests/slot_trace.py``: per seed the number of trace lines and the
    SHA-256 of the trace text (every return value and exception)."""
    import hashlib

    sys.path.insert(0, str(HERE.parent))
    import slot_trace
    from cacheslide_vllm.slide import LayerSlotMap

    seeds = {}
    for seed in range(SLOT_TRACE_SEEDS):
        lines = slot_trace.drive(LayerSlotMap, seed)
        seeds[str(seed)] = dict(lines=len(lines),
                                sha256=hashlib.sha256("\n".join(lines).encode()).hexdigest())
    return dict(steps=120, seeds=seeds)


def main(src: str, only: list[str]) -> None:
    sys.path.insert(0, src)
    import cacheslide_vllm as ref

    torch.set_num_threads(4)
    for name, fn in (("cope", cope_cases), ("wca", wca_cases),
                     ("paged", paged_cases), ("profile", profile_cases)):
        if only and name not in only:
            continue
        cases = fn(ref)
        flat = {f"{case}__{key}": np.asarray(val)
                for case, fields in cases.items() for key, val in fields.items()}
        np.savez_compressed(HERE / f"{name}.npz", **flat)
        print(name, len(flat), "arrays")
    if not only or "slot_trace" in only:
        traces = slot_traces(ref)
        (HERE / "slot_trace.json").write_text(json.dumps(traces, indent=0, sort_keys=True))
        print("slot_trace", len(traces["seeds"]), "seeds")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        raise SystemExit("usage: make_golden.py <CacheSlide checkout>/src "
                         "[cope|wca|paged|profile|slot_trace ...]")
    main(sys.argv[1], sys.argv[2:])
