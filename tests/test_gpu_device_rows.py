"""Active rows on the device and a prefill sized by a device row count.

The next layer's active rows (WCAState.active_indices, wca.py:194-196) and
their association flags (runtime.py:448-454) are produced by
`cs_wca_active_rows` on the device; the tensor-core prefill reads the row
count through `AttnParams.nq_dev`, so the layer's attention runs on the
rows the commit chose without a host read in between.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture
def cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda:0")


@pytest.mark.parametrize("n,extra", [(5000, 17), (4096, 0), (1, 3), (3000, -40)])
def test_active_rows_match_nonzero(cuda, n, extra):
    """rows = nonzero(selected | mandatory) ascending, association = selected
    and not mandatory, -1 / 0 padding to the capacity; a capacity below the
    count keeps the first rows and sets CS_ST_SLOT_RANGE."""
    from cacheslide_b200 import _native as N

    g = torch.Generator().manual_seed(n)
    selected = torch.rand(n, generator=g) < 0.15
    mandatory = torch.zeros(n, dtype=torch.bool)
    mandatory[n // 3: n // 3 + n // 8] = True
    mandatory[n - 1] = True
    selected[n // 3: n // 3 + 10] = True  # some rows both selected and mandatory
    want = torch.nonzero(selected | mandatory).flatten()
    cap = max(len(want) + extra, 0)
    rows = torch.full((max(cap, 1),), 7, dtype=torch.int64, device=cuda)
    assoc = torch.full((max(cap, 1),), 9, dtype=torch.uint8, device=cuda)
    count = torch.full((1,), -5, dtype=torch.int64, device=cuda)
    st = N.Status(cuda)
    lib = N.load()
    sel_d, man_d = selected.to(cuda), mandatory.to(cuda)  # held until the kernel has run
    N.check(lib.cs_wca_active_rows(
        sel_d.data_ptr(), man_d.data_ptr(), n, cap, rows.data_ptr(),
        assoc.data_ptr(), count.data_ptr(), st.ptr, N.stream_of(cuda)), "active_rows")
    torch.cuda.synchronize(cuda)
    got_n = int(count.item())
    assert got_n == min(len(want), cap)
    assert torch.equal(rows[:got_n].cpu(), want[:got_n])
    want_assoc = (selected & ~mandatory)[want[:got_n]].to(torch.uint8)
    assert torch.equal(assoc[:got_n].cpu(), want_assoc)
    assert bool((rows[got_n:cap] == -1).all()) and bool((assoc[got_n:cap] == 0).all())
    assert st.read() == (N.ST_SLOT_RANGE if len(want) > cap else 0)


def test_prefill_rows_from_device_count(cuda):
    """The reuse step's attention over the rows a device-side compaction of
    its commit's masks chose, with the count read by the kernel (nq_dev) and
    the grid sized by a capacity: the same outputs, bit for bit, as the same
    launch given the count on the host; the rows past the count are left as
    they were."""
    from cacheslide_b200 import _native as N
    from cacheslide_b200 import reuse

    cfg = reuse.WorkloadConfig(requests=1, q_heads=8, kv_heads=2, seq=1024, chunks=4, npos=64,
                               fraction=0.15, seed=3)
    work = reuse.SyntheticWorkload(cfg, cuda)
    step = reuse.ReuseStep(work)
    step.run()
    torch.cuda.synchronize(cuda)
    step.check_status()
    r = work.requests[0]
    cap = r.a + 64
    lib = N.load()
    rows = torch.empty(cap, dtype=torch.int64, device=cuda)
    assoc = torch.empty(cap, dtype=torch.uint8, device=cuda)
    count = torch.empty(1, dtype=torch.int64, device=cuda)
    st = N.Status(cuda)
    s = N.stream_of(cuda)
    N.check(lib.cs_wca_active_rows(r.selected.data_ptr(), r.mandatory.data_ptr(), cfg.seq, cap,
                                   rows.data_ptr(), assoc.data_ptr(), count.data_ptr(), st.ptr,
                                   s), "active_rows")
    # the layer's inputs for those rows, gathered on the device (no host read)
    idx = rows.clamp_min(0)
    q = r.q_all.index_select(0, idx).contiguous()
    co = r.offsets.index_select(1, idx).contiguous()
    outs = []
    for device_count in (True, False):
        out = torch.full((cap, cfg.q_heads, cfg.head_dim), 3.0, dtype=cfg.dtype, device=cuda)
        p = step._attn_params(r)
        p.q = q.data_ptr()
        p.q_stride_tok, p.q_stride_head = q.stride(0), q.stride(1)
        p.qpos = rows.data_ptr()
        p.q_selected = assoc.data_ptr()
        p.chunk_off = co.data_ptr()
        p.co_stride_h, p.co_stride_q = co.stride(0), co.stride(1)
        p.out = out.data_ptr()
        p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
        p.status = st.ptr
        if device_count:
            p.nq = cap
            p.nq_dev = count.data_ptr()
        else:
            torch.cuda.synchronize(cuda)
            p.nq = int(count.item())
        N.check(lib.cs_cope_attn_prefill(ctypes.byref(p), s), "prefill")
        torch.cuda.synchronize(cuda)
        assert st.read() == 0
        outs.append(out.cpu())
    nlive = int(count.item())
    assert nlive == int((r.selected | r.mandatory).sum().item())
    assert torch.equal(outs[0][:nlive], outs[1][:nlive])
    assert bool((outs[0][nlive:] == 3.0).all())
    # the other attention entry points refuse a device row count
    p = step._attn_params(r)
    p.nq_dev = count.data_ptr()
    assert lib.cs_cope_attn(ctypes.byref(p), s) == N.CS_ERR_UNSUPPORTED


def test_wca_state_active_rows_device(cuda):
    """WCAState.active_rows_device equals active_indices after a commit."""
    from cacheslide_b200 import wca as W

    g = torch.Generator().manual_seed(5)
    n, hkv, d = 2000, 2, 64
    cached = (torch.randn(n, hkv, d, generator=g) / 8).to(torch.bfloat16).to(cuda)
    fresh = (cached.float().cpu() + 0.05 * torch.randn(n, hkv, d, generator=g)).to(
        torch.bfloat16).to(cuda)
    reused = torch.ones(n, dtype=torch.bool)
    reused[500:700] = False
    mandatory = ~reused
    mandatory[n - 1] = True
    st = W.WCAState.initialize(cached, fresh, reused.to(cuda), mandatory.to(cuda))
    rows, assoc, count = st.active_rows_device(n)
    torch.cuda.synchronize(cuda)
    want = st.active_indices
    k = int(count.item())
    assert k == want.numel()
    assert torch.equal(rows[:k], want)
    want_assoc = (st.selected_mask & ~st.mandatory_mask)[want].to(torch.uint8)
    assert torch.equal(assoc[:k], want_assoc)


def test_layer_chained_on_device_rows(cuda):
    """Layer 2 of a reuse step run from the rows layer 1's commit chose, with
    no host read: the active rows on the device, the WCA update (blend and
    paged scatter) and commit with the device row count (a_dev), and the
    attention with nq_dev, every launch sized by a capacity.  Against the
    same layer given the count on the host, from the same saved state: the
    paged cache bytes, weights, masks, removal and promotion lists, cosines
    and attention outputs are equal bit for bit."""
    from cacheslide_b200 import _native as N
    from cacheslide_b200 import reuse

    cfg = reuse.WorkloadConfig(requests=1, q_heads=8, kv_heads=2, seq=1024, chunks=4, npos=64,
                               fraction=0.15, seed=9)
    work = reuse.SyntheticWorkload(cfg, cuda)
    step = reuse.ReuseStep(work, batched=True)
    step.run()  # layer 1: its commit decides layer 2's rows
    torch.cuda.synchronize(cuda)
    step.check_status()
    r = work.requests[0]
    n, hkv, d, hq = cfg.seq, cfg.kv_heads, cfg.head_dim, cfg.q_heads
    g = torch.Generator().manual_seed(21)
    fresh_k2 = (r.cached_k.float().cpu() + 0.05 * torch.randn(n, hkv, d, generator=g)).to(
        cfg.dtype).to(cuda)
    fresh_v2 = (r.cached_v.float().cpu() + 0.05 * torch.randn(n, hkv, d, generator=g)).to(
        cfg.dtype).to(cuda)
    q2 = (torch.randn(n, hq, d, generator=g) / d ** 0.5).to(cfg.dtype).to(cuda)
    lib = N.load()
    s = N.stream_of(cuda)
    cap = r.a + 128
    state = [r.alpha, r.candidate, r.selected, r.removed]
    saved = [t.clone() for t in state] + [work.cache.clone()]

    def layer2(device: bool):
        st = N.Status(cuda)
        rows = torch.empty(cap, dtype=torch.int64, device=cuda)
        assoc = torch.empty(cap, dtype=torch.uint8, device=cuda)
        count = torch.empty(1, dtype=torch.int64, device=cuda)
        N.check(lib.cs_wca_active_rows(r.selected.data_ptr(), r.mandatory.data_ptr(), n, cap,
                                       rows.data_ptr(), assoc.data_ptr(), count.data_ptr(),
                                       st.ptr, s), "active_rows")
        if device:
            a, a_dev = cap, count.data_ptr()
        else:
            torch.cuda.synchronize(cuda)
            a, a_dev = int(count.item()), None
        idx = rows[:a].clamp_min(0)
        fk, fv = fresh_k2.index_select(0, idx), fresh_v2.index_select(0, idx)
        slots = r.slots.index_select(0, idx)
        nxt = torch.empty(a, dtype=torch.float64, device=cuda)
        used = torch.empty_like(nxt)
        cos = torch.empty_like(nxt)
        upd = (N.UpdateItem * 1)(N.UpdateItem(
            r.cached_k.data_ptr(), r.cached_v.data_ptr(), r.cached_k.stride(0),
            r.cached_k.stride(1), fk.data_ptr(), fv.data_ptr(), fk.stride(0), fk.stride(1),
            rows.data_ptr(), a, r.alpha.data_ptr(), r.mandatory.data_ptr(), None, None,
            nxt.data_ptr(), used.data_ptr(), cos.data_ptr(), slots.data_ptr(), st.ptr, a_dev))
        N.check(lib.cs_wca_update_batch(upd, 1, hkv, d, N.DTYPES[cfg.dtype], 0, 1e-8, 0,
                                        ctypes.byref(step.kv), s), "update")
        q = q2.index_select(0, idx)
        co = r.offsets.index_select(1, idx).contiguous()
        out = torch.full((a, hq, d), 3.0, dtype=cfg.dtype, device=cuda)
        p = step._attn_params(r)
        p.q = q.data_ptr()
        p.q_stride_tok, p.q_stride_head = q.stride(0), q.stride(1)
        p.nq = a
        p.nq_dev = a_dev
        p.qpos = rows.data_ptr()
        p.q_selected = assoc.data_ptr()
        p.chunk_off = co.data_ptr()
        p.co_stride_h, p.co_stride_q = co.stride(0), co.stride(1)
        p.out = out.data_ptr()
        p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
        p.status = st.ptr
        N.check(lib.cs_cope_attn_prefill(ctypes.byref(p), s), "prefill")
        removed_list = torch.full((n,), -7, dtype=torch.int64, device=cuda)
        promoted = torch.full((n,), -7, dtype=torch.int64, device=cuda)
        counts = torch.zeros(2, dtype=torch.int64, device=cuda)
        com = (N.CommitItem * 1)(N.CommitItem(
            rows.data_ptr(), a, nxt.data_ptr(), cos.data_ptr(), n, r.budget, r.dev.data_ptr(),
            r.alpha.data_ptr(), r.candidate.data_ptr(), r.selected.data_ptr(),
            r.removed.data_ptr(), removed_list.data_ptr(), promoted.data_ptr(),
            counts.data_ptr(), st.ptr, a_dev))
        N.check(lib.cs_wca_commit_batch(com, 1, 0.12, 0, s), "commit")
        torch.cuda.synchronize(cuda)
        assert st.read() == 0
        k = int(count.item())
        nr, npr = counts.tolist()
        return {"count": k, "out": out[:k].cpu(), "next": nxt[:k].cpu(), "cos": cos[:k].cpu(),
                "alpha": r.alpha.cpu(), "candidate": r.candidate.cpu(),
                "selected": r.selected.cpu(), "removed": r.removed.cpu(),
                "removed_list": removed_list[:nr].cpu(), "promoted": promoted[:npr].cpu(),
                "counts": (nr, npr), "cache": work.cache.cpu(),
                "untouched": bool((out[k:] == 3.0).all()) if device else True}

    got = layer2(True)
    for t, v in zip(state + [work.cache], saved):
        t.copy_(v)
    want = layer2(False)
    assert got["count"] == want["count"] and got["count"] > 0
    assert got["untouched"]
    for key in ("out", "next", "cos", "alpha", "candidate", "selected", "removed",
                "removed_list", "promoted", "cache"):
        assert torch.equal(got[key], want[key]), key
    assert got["counts"] == want["counts"]


def test_qkv_rows_from_device_count(cuda):
    """The selective QKV GEMM (cs_qkv_gather_lora) over rows listed on the
    device, with the row count read from device memory (a_dev) and the grid
    sized by a capacity: bit for bit the launch given the count on the host;
    the output rows past the count are not written."""
    from cacheslide_b200 import _native as N

    g = torch.Generator().manual_seed(4)
    n, hidden, n_out, rank = 1500, 512, 512, 16
    dt = torch.bfloat16
    src = (torch.randn(n, hidden, generator=g)).to(dt).to(cuda)
    w = (torch.randn(n_out, hidden, generator=g) / hidden ** 0.5).to(dt).to(cuda)
    la = (torch.randn(rank, hidden, generator=g) / hidden ** 0.5).to(dt).to(cuda)
    lb = (torch.randn(n_out, rank, generator=g) * 0.5).to(dt).to(cuda)
    selected = (torch.rand(n, generator=g) < 0.2).to(cuda)
    mandatory = torch.zeros(n, dtype=torch.bool, device=cuda)
    mandatory[600:700] = True
    cap = 700
    lib = N.load()
    s = N.stream_of(cuda)
    st = N.Status(cuda)
    rows = torch.empty(cap, dtype=torch.int64, device=cuda)
    assoc = torch.empty(cap, dtype=torch.uint8, device=cuda)
    count = torch.empty(1, dtype=torch.int64, device=cuda)
    N.check(lib.cs_wca_active_rows(selected.data_ptr(), mandatory.data_ptr(), n, cap,
                                   rows.data_ptr(), assoc.data_ptr(), count.data_ptr(), st.ptr, s),
            "active_rows")
    row_src = torch.zeros(cap, dtype=torch.int32, device=cuda)
    outs = []
    for device_count in (True, False):
        out = torch.full((cap, n_out), 5.0, dtype=dt, device=cuda)
        p = N.QKVParams()
        p.src0, p.src0_stride, p.src0_rows = src.data_ptr(), src.stride(0), n
        p.src1, p.src1_stride, p.src1_rows = src.data_ptr(), src.stride(0), n
        p.row_src, p.row_idx = row_src.data_ptr(), rows.data_ptr()
        p.hidden, p.n_out = hidden, n_out
        p.w, p.lora_a, p.lora_b, p.rank = w.data_ptr(), la.data_ptr(), lb.data_ptr(), rank
        p.out, p.out_stride = out.data_ptr(), out.stride(0)
        p.dtype = N.DTYPES[dt]
        p.status = st.ptr
        if device_count:
            p.a, p.a_dev = cap, count.data_ptr()
        else:
            torch.cuda.synchronize(cuda)
            p.a = int(count.item())
        N.check(lib.cs_qkv_gather_lora(ctypes.byref(p), s), "qkv")
        torch.cuda.synchronize(cuda)
        assert st.read() == 0
        outs.append(out.cpu())
    k = int(count.item())
    assert 0 < k < cap
    assert torch.equal(outs[0][:k], outs[1][:k])
    assert bool((outs[0][k:] == 5.0).all())


def test_chained_layers_match_host_count_layers(cuda):
    """chain.ChainedLayers: layers 2-4 of a request, each on the rows the
    previous layer's commit chose, with no host read between layers, equal
    bit for bit to the same layers with the count read back to the host
    before each (the reference runtime's order, runtime.py:410): the final
    WCA state, the last layer's attention rows and the paged cache."""
    from cacheslide_b200 import reuse
    from cacheslide_b200.chain import ChainedLayers

    cfg = reuse.WorkloadConfig(requests=1, q_heads=8, kv_heads=2, seq=1024, chunks=4, npos=64,
                               fraction=0.15, seed=12)
    work = reuse.SyntheticWorkload(cfg, cuda)
    step = reuse.ReuseStep(work, batched=True)
    step.run()
    torch.cuda.synchronize(cuda)
    step.check_status()
    r = work.requests[0]
    chain = ChainedLayers(step, layers=4)
    state = [r.alpha, r.candidate, r.selected, r.removed, work.cache]
    saved = [t.clone() for t in state]
    results = []
    for device in (True, False):
        for t, v in zip(state, saved):
            t.copy_(v)
        chain.run(device=device)
        torch.cuda.synchronize(cuda)
        step.check_status()
        k = int(chain.count.item())
        results.append({"k": k, "out": chain.out[:k].cpu(), "alpha": r.alpha.cpu(),
                        "candidate": r.candidate.cpu(), "selected": r.selected.cpu(),
                        "removed": r.removed.cpu(), "cache": work.cache.cpu()})
    got, want = results
    assert got["k"] == want["k"] > 0
    for key in ("out", "alpha", "candidate", "selected", "removed", "cache"):
        assert torch.equal(got[key], want[key]), key
