"""Batched launches of a step's per-request calls (cs_slide_scatter_batch,
cs_wca_initialize_batch / update_batch / commit_batch): bit-identical to the
single calls they replace (the reference runs one call per request,
paged.py:205-240 and wca.py:152-366).

* the whole reuse step in batched mode (seven launches for all requests)
  against the default per-request mode on identical inputs: WCA state,
  paged cache bytes and attention outputs equal bit for bit, at three head
  layouts (8, 2 and 1 KV heads of 128: register-resident rows of four, one
  and -- for one head -- the half-warp vector path);
* direct batched calls with ragged items (different lengths, an empty item,
  row selections) against one single call per item.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _state(step):
    out = []
    for r in step.work.requests:
        out.append({k: getattr(r, k).clone() for k in (
            "dev", "alpha", "candidate", "selected", "removed", "counts", "counts2",
            "next_alpha", "used_alpha", "cos", "out")})
        out[-1]["promoted"] = r.promoted[: int(r.counts2[1])].clone()
        out[-1]["removed_list"] = r.removed_list[: int(r.counts2[0])].clone()
    return out


@pytest.mark.parametrize("kv_heads,q_heads", [(8, 32), (2, 8), (1, 8)])
def test_batched_step_equals_per_request_step(cuda, kv_heads, q_heads):
    from cacheslide_b200 import reuse

    cfg = reuse.WorkloadConfig(requests=3, q_heads=q_heads, kv_heads=kv_heads, head_dim=128,
                               seq=1024, chunks=4, npos=64, block=16, fraction=0.15, seed=9)
    runs = []
    for batched in (False, True):
        work = reuse.SyntheticWorkload(cfg, cuda)
        step = reuse.ReuseStep(work, batched=batched)
        step.run()
        torch.cuda.synchronize()
        step.check_status()
        runs.append((work, step, _state(step)))
    (w0, s0, a), (w1, s1, b) = runs
    assert torch.equal(w0.requests[0].cached_k, w1.requests[0].cached_k)  # same inputs
    for i, (x, y) in enumerate(zip(a, b)):
        for key in x:
            assert torch.equal(x[key], y[key]), f"request {i}: {key}"
    # every record the step wrote: snapshot plus fused rows
    assert torch.equal(w0.cache.view(torch.int16), w1.cache.view(torch.int16))
    assert all(int(x["selected"].sum()) > 0 for x in b)  # a selection was made


def test_batched_calls_match_single_calls_with_ragged_items(cuda):
    from cacheslide_b200 import _native as N

    lib = N.load()
    g = torch.Generator(device="cpu").manual_seed(3)
    heads, dim, bs = 4, 64, 16
    sizes = [300, 0, 77, 513]
    dt = torch.bfloat16

    def rnd(*shape):
        return torch.randn(*shape, generator=g).to(dt).to(cuda)

    cached = [rnd(n, heads, dim) for n in sizes]
    fresh = [c + 0.1 * rnd(*c.shape) for c in cached]
    # outputs and masks hold at least one element: the calls take non-NULL
    # pointers even for an empty item
    reused = [(torch.rand(max(n, 1), generator=g) < 0.8).to(cuda) for n in sizes]
    s = N.stream_of(cuda)

    def init_outputs():
        return [dict(dev=torch.full((max(n, 1),), -1.0, dtype=torch.float64, device=cuda),
                     alpha=torch.full((max(n, 1),), -1.0, dtype=torch.float64, device=cuda),
                     cand=torch.full((max(n, 1),), 7, dtype=torch.bool, device=cuda),
                     sel=torch.ones(max(n, 1), dtype=torch.bool, device=cuda),
                     rem=torch.ones(max(n, 1), dtype=torch.bool, device=cuda),
                     counts=torch.full((2,), 99, dtype=torch.int64, device=cuda),
                     st=torch.zeros(1, dtype=torch.int32, device=cuda)) for n in sizes]

    single, batch = init_outputs(), init_outputs()
    for i, n in enumerate(sizes):
        o = single[i]
        N.check(lib.cs_wca_initialize(
            cached[i].data_ptr(), cached[i].stride(0), cached[i].stride(1), fresh[i].data_ptr(),
            fresh[i].stride(0), fresh[i].stride(1), n, heads, dim, N.CS_BF16,
            reused[i].data_ptr(), 1e-8, 0, o["dev"].data_ptr(), o["alpha"].data_ptr(),
            o["cand"].data_ptr(), o["sel"].data_ptr(), o["rem"].data_ptr(),
            o["counts"].data_ptr(), o["st"].data_ptr(), s), "single initialize")
    items = (N.InitializeItem * len(sizes))(*[N.InitializeItem(
        cached[i].data_ptr(), cached[i].stride(0), cached[i].stride(1), fresh[i].data_ptr(),
        fresh[i].stride(0), fresh[i].stride(1), n, reused[i].data_ptr(),
        batch[i]["dev"].data_ptr(), batch[i]["alpha"].data_ptr(), batch[i]["cand"].data_ptr(),
        batch[i]["sel"].data_ptr(), batch[i]["rem"].data_ptr(), batch[i]["counts"].data_ptr(),
        batch[i]["st"].data_ptr()) for i, n in enumerate(sizes)])
    N.check(lib.cs_wca_initialize_batch(items, len(sizes), heads, dim, N.CS_BF16, 1e-8, 0, s),
            "batched initialize")
    torch.cuda.synchronize()
    for i in range(len(sizes)):
        for key in single[i]:
            assert torch.equal(single[i][key], batch[i][key]), f"initialize item {i}: {key}"
    assert int(batch[1]["counts"].abs().sum()) == 0  # the empty item's counts are zeroed

    # update: active rows of each item (one item without rows), paged writes
    nblocks = sum((n + bs - 1) // bs for n in sizes) + 2
    pools = [torch.zeros(nblocks, heads, bs, 2 * dim, dtype=dt, device=cuda) for _ in range(2)]
    perm = torch.randperm(nblocks * bs, generator=g).to(cuda)
    act, slots, fk, fv, cv, base = [], [], [], [], [], 0
    for i, n in enumerate(sizes):
        a = 0 if i == 1 else max(1, n // 3)
        idx = torch.sort(torch.randperm(max(n, 1), generator=g)[:a]).values.to(cuda)
        act.append(idx)
        slots.append(perm[base:base + a].contiguous())
        base += a
        fk.append(rnd(a, heads, dim))
        fv.append(rnd(a, heads, dim))
        cv.append(rnd(n, heads, dim))
    mand = [(torch.rand(n, generator=g) < 0.2).to(cuda) for n in sizes]

    def upd_outputs():
        return [dict(nxt=torch.zeros(a.numel(), dtype=torch.float64, device=cuda),
                     used=torch.zeros(a.numel(), dtype=torch.float64, device=cuda),
                     cos=torch.zeros(a.numel(), dtype=torch.float64, device=cuda),
                     fk=torch.zeros(a.numel(), heads, dim, dtype=dt, device=cuda),
                     fv=torch.zeros(a.numel(), heads, dim, dtype=dt, device=cuda),
                     st=torch.zeros(1, dtype=torch.int32, device=cuda)) for a in act]

    us, ub = upd_outputs(), upd_outputs()
    kvs = [N.paged_view(p) for p in pools]
    for i in range(len(sizes)):
        o = us[i]
        N.check(lib.cs_wca_update(
            cached[i].data_ptr(), cv[i].data_ptr(), cached[i].stride(0), cached[i].stride(1),
            fk[i].data_ptr(), fv[i].data_ptr(), fk[i].stride(0), fk[i].stride(1),
            act[i].data_ptr(), act[i].numel(), heads, dim, N.CS_BF16, single[i]["alpha"].data_ptr(),
            mand[i].data_ptr(), 0, 1e-8, 0, o["fk"].data_ptr(), o["fv"].data_ptr(),
            o["nxt"].data_ptr(), o["used"].data_ptr(), o["cos"].data_ptr(),
            ctypes.byref(kvs[0]), slots[i].data_ptr(), o["st"].data_ptr(), s), "single update")
    uitems = (N.UpdateItem * len(sizes))(*[N.UpdateItem(
        cached[i].data_ptr(), cv[i].data_ptr(), cached[i].stride(0), cached[i].stride(1),
        fk[i].data_ptr(), fv[i].data_ptr(), fk[i].stride(0), fk[i].stride(1), act[i].data_ptr(),
        act[i].numel(), batch[i]["alpha"].data_ptr(), mand[i].data_ptr(), ub[i]["fk"].data_ptr(),
        ub[i]["fv"].data_ptr(), ub[i]["nxt"].data_ptr(), ub[i]["used"].data_ptr(),
        ub[i]["cos"].data_ptr(), slots[i].data_ptr(), ub[i]["st"].data_ptr())
        for i in range(len(sizes))])
    N.check(lib.cs_wca_update_batch(uitems, len(sizes), heads, dim, N.CS_BF16, 0, 1e-8, 0,
                                    ctypes.byref(kvs[1]), s), "batched update")
    torch.cuda.synchronize()
    for i in range(len(sizes)):
        for key in us[i]:
            assert torch.equal(us[i][key].view(-1).view(torch.uint8),
                               ub[i][key].view(-1).view(torch.uint8)), f"update item {i}: {key}"
    assert torch.equal(pools[0].view(torch.int16), pools[1].view(torch.int16))

    # commit with removals and promotions, one block per item
    def commit_state(src):
        return [dict(alpha=src[i]["alpha"].clone(), cand=src[i]["cand"].clone(),
                     sel=src[i]["sel"].clone(), rem=src[i]["rem"].clone(),
                     rl=torch.full((max(n, 1),), -1, dtype=torch.int64, device=cuda),
                     pr=torch.full((max(n, 1),), -1, dtype=torch.int64, device=cuda),
                     counts=torch.zeros(2, dtype=torch.int64, device=cuda),
                     st=torch.zeros(1, dtype=torch.int32, device=cuda))
                for i, n in enumerate(sizes)]

    cs_, cb = commit_state(single), commit_state(batch)
    for i in range(len(sizes)):  # the active rows are selected: the gate can remove them
        if act[i].numel():
            cs_[i]["sel"][act[i]] = True
            cb[i]["sel"][act[i]] = True
    budgets = [max(1, n // 4) for n in sizes]
    for i, n in enumerate(sizes):
        o = cs_[i]
        N.check(lib.cs_wca_commit(
            act[i].data_ptr() if act[i].numel() else None, act[i].numel(),
            us[i]["nxt"].data_ptr(), us[i]["cos"].data_ptr(), 0.99, 0, n, budgets[i],
            single[i]["dev"].data_ptr(), o["alpha"].data_ptr(), o["cand"].data_ptr(),
            o["sel"].data_ptr(), o["rem"].data_ptr(), o["rl"].data_ptr(), o["pr"].data_ptr(),
            o["counts"].data_ptr(), o["st"].data_ptr(), s), "single commit")
    citems = (N.CommitItem * len(sizes))(*[N.CommitItem(
        act[i].data_ptr() if act[i].numel() else None, act[i].numel(), ub[i]["nxt"].data_ptr(),
        ub[i]["cos"].data_ptr(), n, budgets[i], batch[i]["dev"].data_ptr(),
        cb[i]["alpha"].data_ptr(), cb[i]["cand"].data_ptr(), cb[i]["sel"].data_ptr(),
        cb[i]["rem"].data_ptr(), cb[i]["rl"].data_ptr(), cb[i]["pr"].data_ptr(),
        cb[i]["counts"].data_ptr(), cb[i]["st"].data_ptr()) for i, n in enumerate(sizes)])
    N.check(lib.cs_wca_commit_batch(citems, len(sizes), 0.99, 0, s), "batched commit")
    torch.cuda.synchronize()
    for i in range(len(sizes)):
        for key in cs_[i]:
            assert torch.equal(cs_[i][key], cb[i][key]), f"commit item {i}: {key}"
    assert sum(int(c["counts"][0]) for c in cb) > 0  # removals happened

    # scatter: rows selections and an empty item into two pools
    pools = [torch.zeros(nblocks, heads, bs, 2 * dim, dtype=dt, device=cuda) for _ in range(2)]
    kvs = [N.paged_view(p) for p in pools]
    rows = [torch.randperm(max(n, 1), generator=g)[: n // 2].to(cuda) for n in sizes]
    sl, base = [], 0
    for r in rows:
        sl.append(perm[base:base + r.numel()].contiguous())
        base += r.numel()
    st = torch.zeros(2, dtype=torch.int32, device=cuda)
    for i in range(len(sizes)):
        N.check(lib.cs_slide_scatter(
            ctypes.byref(kvs[0]), sl[i].data_ptr(), rows[i].data_ptr(), rows[i].numel(),
            cached[i].data_ptr(), cv[i].data_ptr(), cached[i].stride(0), cached[i].stride(1),
            st[0:1].data_ptr(), s), "single scatter")
    sitems = (N.ScatterItem * len(sizes))(*[N.ScatterItem(
        sl[i].data_ptr(), rows[i].data_ptr(), rows[i].numel(), cached[i].data_ptr(),
        cv[i].data_ptr(), cached[i].stride(0), cached[i].stride(1), st[1:2].data_ptr())
        for i in range(len(sizes))])
    N.check(lib.cs_slide_scatter_batch(ctypes.byref(kvs[1]), sitems, len(sizes), s),
            "batched scatter")
    torch.cuda.synchronize()
    assert st.tolist() == [0, 0]
    assert torch.equal(pools[0].view(torch.int16), pools[1].view(torch.int16))
    assert int(pools[1].view(torch.int16).abs().sum()) > 0
