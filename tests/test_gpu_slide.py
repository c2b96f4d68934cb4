"""SLIDE paged KV kernels and NativePagedKV on the GPU: bit-exact parity.

Raw bytes are compared through integer views, so every assertion here is
exact.  Scenarios restate the reference's tests/test_paged.py (strided
non-contiguous cache, permuted block table, exact slot numbers) plus the
golden arena produced by the reference itself.
"""

from __future__ import annotations

import ctypes
import json
from concurrent.futures import Future

import numpy as np
import pytest
import torch

from cacheslide_b200 import _native as N
from cacheslide_b200.paged import NativePagedKV
from oracle import slide as oslide
from tests.conftest import golden

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> np.ndarray:
    view = {2: torch.int16, 4: torch.int32, 8: torch.int64}[t.element_size()]
    return t.detach().contiguous().view(view).cpu().numpy()


def _rand_cache(nb, hkv, bs, d, dtype, device, strided=False, seed=0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    if strided:
        backing = torch.randn(nb, hkv, bs, 4 * d, generator=g).to(dtype).to(device)
        return backing[..., ::2], backing
    c = torch.randn(nb, hkv, bs, 2 * d, generator=g).to(dtype).to(device)
    return c, c


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32, torch.float64])
@pytest.mark.parametrize("strided", [False, True])
def test_gather_scatter_relocate_bit_exact(cuda, dtype, strided):
    nb, hkv, bs, d, side = 37, 4, 16, 64, 23
    cache, _ = _rand_cache(nb, hkv, bs, d, dtype, cuda, strided)
    side_k = torch.randn(side, hkv, d).to(dtype).to(cuda)
    side_v = torch.randn(side, hkv, d).to(dtype).to(cuda)
    rng = np.random.default_rng(1)
    total = nb * bs + side
    slots = rng.permutation(total)[:300]
    kv = N.paged_view(cache, side_k, side_v)
    lib = N.load()
    st = N.Status(cuda)
    # gather
    s_t = torch.from_numpy(slots).to(cuda)
    ok = torch.empty(len(slots), hkv, d, dtype=dtype, device=cuda)
    ov = torch.empty_like(ok)
    N.check(lib.cs_slide_gather(ctypes.byref(kv), s_t.data_ptr(), len(slots), ok.data_ptr(),
                                ov.data_ptr(), ok.stride(0), ok.stride(1), st.ptr,
                                N.stream_of(cuda)), "gather")
    ek, ev = oslide.gather(_bits(cache), _bits(side_k), _bits(side_v), slots)
    np.testing.assert_array_equal(_bits(ok), ek)
    np.testing.assert_array_equal(_bits(ov), ev)
    # scatter with a row selection
    src_k = torch.randn(500, hkv, d).to(dtype).to(cuda)
    src_v = torch.randn(500, hkv, d).to(dtype).to(cuda)
    rows = rng.integers(0, 500, len(slots))
    r_t = torch.from_numpy(rows).to(cuda)
    host = [_bits(cache).copy(), _bits(side_k).copy(), _bits(side_v).copy()]
    N.check(lib.cs_slide_scatter(ctypes.byref(kv), s_t.data_ptr(), r_t.data_ptr(), len(slots),
                                 src_k.data_ptr(), src_v.data_ptr(), src_k.stride(0),
                                 src_k.stride(1), st.ptr, N.stream_of(cuda)), "scatter")
    oslide.scatter(*host, slots, _bits(src_k)[rows], _bits(src_v)[rows])
    np.testing.assert_array_equal(_bits(cache), host[0])
    np.testing.assert_array_equal(_bits(side_k), host[1])
    # relocate disjoint slot sets
    perm = rng.permutation(total)
    src, dst = perm[:100], perm[100:200]
    a, b = torch.from_numpy(src).to(cuda), torch.from_numpy(dst).to(cuda)
    N.check(lib.cs_slide_relocate(ctypes.byref(kv), a.data_ptr(), b.data_ptr(), 100, st.ptr,
                                  N.stream_of(cuda)), "relocate")
    oslide.relocate(*host, src, dst)
    np.testing.assert_array_equal(_bits(cache), host[0])
    np.testing.assert_array_equal(_bits(side_v), host[2])
    assert st.read() == 0


def test_out_of_range_slot_sets_status_and_skips(cuda):
    cache, _ = _rand_cache(4, 2, 4, 16, torch.bfloat16, cuda)
    before = _bits(cache).copy()
    kv = N.paged_view(cache)
    slots = torch.tensor([1, 16, -3, 5], device=cuda)
    k = torch.ones(4, 2, 16, dtype=torch.bfloat16, device=cuda)
    st = N.Status(cuda)
    N.check(N.load().cs_slide_scatter(ctypes.byref(kv), slots.data_ptr(), None, 4, k.data_ptr(),
                                      k.data_ptr(), k.stride(0), k.stride(1), st.ptr,
                                      N.stream_of(cuda)), "scatter")
    assert st.read() & N.ST_SLOT_RANGE
    after = _bits(cache)
    # changed (block, offset) pairs, flattened to slot numbers: only 1 and 5
    changed = np.nonzero((after != before).any(axis=(1, 3)).reshape(-1))[0]
    assert set(changed.tolist()) == {1, 5}


def _fixture_arena(cuda, max_selected=2):
    backing = torch.full((8, 2, 2, 12), -999.0, device=cuda)
    cache = backing[..., ::2]
    assert not cache.is_contiguous()
    arena = NativePagedKV(cache, [4, 1, 6, 3], 5, max_selected, request_id="a", layer_index=2)
    key = torch.arange(30, dtype=cache.dtype, device=cuda).reshape(5, 2, 3) / 30
    value = key + 10
    arena.write_prefill(key, value)
    return arena, key, value, backing


def test_arena_noncontiguous_staged_wca_decode(cuda):
    """reference tests/test_paged.py:245-311 restated on the device."""
    arena, key, value, backing = _fixture_arena(cuda)
    assert arena.snapshot() == {0: 8, 1: 9, 2: 2, 3: 3, 4: 12}
    loading = Future()
    sel = torch.tensor([3, 1])
    mapping = arena.promote_selected(sel, key[sel] + 1, value[sel] + 2,
                                     load_future=loading).result()
    assert mapping[3] == 16 and mapping[1] == 17
    assert arena.stats()["vacated_slots"] == 2
    with pytest.raises(RuntimeError, match="load must complete"):
        arena.write_prefill(key, value)
    loading.set_result(None)
    arena.write_prefill(key, value)
    upd = [1, 3, 4]
    fk, fv = key[upd] + 0.5, value[upd] + 0.75
    arena.update_selected(upd, fk, fv)
    key[upd], value[upd] = fk, fv
    order = [4, 1, 0, 3, 2]
    gk, gv = arena.gather(order)
    assert torch.equal(gk, key[order]) and torch.equal(gv, value[order])
    assert arena.decode(5, key[0] + 2, value[0] + 2, 13) == 3
    assert arena.decode(6, key[0] + 3, value[0] + 3, 6) == 9
    assert arena.decode(7, key[0] + 4, value[0] + 4, 7) == 7
    ek = torch.cat((key, key[:1] + 2, key[:1] + 3, key[:1] + 4))
    gk, _ = arena.gather(range(8))
    assert torch.equal(gk, ek)
    assert torch.all(arena.cache[0] == -999)
    assert torch.all(backing[..., 1::2] == -999)
    assert arena.stats()["physical_hole_reuse"] == 2
    assert arena.stats()["decode_native_bind"] == 1


def test_arena_matches_reference_golden_bytes(cuda):
    a = golden("paged")["arena"]
    nb, hkv, bs, d2 = a["cache"].shape
    cache = torch.zeros(nb, hkv, bs, d2, dtype=torch.bfloat16, device=cuda)
    arena = NativePagedKV(cache, a["table"].tolist(), 18, 4, request_id="g", layer_index=1)
    key = torch.from_numpy(a["key"]).view(torch.bfloat16).to(cuda)
    value = torch.from_numpy(a["value"]).view(torch.bfloat16).to(cuda)
    arena.write_prefill(key, value)
    assert [arena.snapshot()[t] for t in range(18)] == a["snap0"].tolist()
    loading = Future()
    sel = [3, 11, 6]
    m1 = arena.promote_selected(sel, key[sel] + 1, value[sel] - 1, load_future=loading).result()
    assert [m1[t] for t in sel] == a["promoted"].tolist()
    loading.set_result(None)
    arena.write_prefill(key, value)
    upd = [3, 6, 11, 17]
    arena.update_selected(upd, key[upd] * 2, value[upd] * 3)
    d1 = arena.decode(18, key[0] + 5, value[0] + 5)
    d2 = arena.decode(19, key[1] + 6, value[1] + 6)
    assert [d1, d2] == a["decode"].tolist()
    assert [arena.snapshot()[t] for t in range(20)] == a["final_map"].tolist()
    gk, gv = arena.gather(a["order"].tolist())
    np.testing.assert_array_equal(_bits(gk), a["gathered_k"])
    np.testing.assert_array_equal(_bits(gv), a["gathered_v"])
    np.testing.assert_array_equal(_bits(cache), a["cache"])
    # the sidecar is allocated uninitialised (paged.py:227-232): compare the
    # rows the three promotions wrote
    written = [s - nb * bs for s in a["promoted"].tolist()]
    np.testing.assert_array_equal(_bits(arena._side_key)[written], a["side_k"][written])
    np.testing.assert_array_equal(_bits(arena._side_value)[written], a["side_v"][written])
    assert arena.stats() == json.loads(str(a["stats"]))


def test_ready_inplace_branch_keeps_native_slots(cuda):
    """reference tests/test_paged.py:34-55."""
    arena, key, value, _ = _fixture_arena(cuda, max_selected=0)
    original = arena.snapshot()
    assert arena.write_selected_ready([1, 3], key[[1, 3]] + 1, value[[1, 3]] + 2) == original
    key[[1, 3]] += 1
    value[[1, 3]] += 2
    gk, gv = arena.gather(range(5))
    assert torch.equal(gk, key) and torch.equal(gv, value)
    assert arena.stats()["sidecar_allocated_slots"] == 0
    assert arena.decode(5, key[0], value[0]) == 13
