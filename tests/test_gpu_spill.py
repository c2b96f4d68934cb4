"""Dirty-page writeback: page images (cs_slide_pack_pages / unpack) and
NativePagedKV.spill / reload, bit-exact.

The reference only advises a spill order (paged.py:530-559: clean pages
first, then more selected tokens, guarded pages excluded); here the pages of
that order are packed on the device into native-block images, copied to
pinned host memory with the pages' slots pinned until the copy lands, and
can be written back.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from cacheslide_b200 import _native as N
from tests.test_gpu_slide import _bits, _fixture_arena

pytestmark = pytest.mark.gpu


def _image(cache, side_k, side_v, page, bs):
    """The image of one page built by plain indexing: [heads, bs, 2D]."""
    nb = cache.shape[0]
    if page < nb:
        return cache[page].clone()
    hkv, d = cache.shape[1], cache.shape[3] // 2
    img = torch.zeros(hkv, bs, 2 * d, dtype=cache.dtype, device=cache.device)
    first = (page - nb) * bs
    rows = max(0, min(bs, side_k.shape[0] - first))
    img[:, :rows, :d] = side_k[first:first + rows].transpose(0, 1)
    img[:, :rows, d:] = side_v[first:first + rows].transpose(0, 1)
    return img


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_pack_unpack_pages_round_trip(cuda, dtype):
    nb, hkv, bs, d, side = 37, 4, 16, 64, 23
    g = torch.Generator().manual_seed(3)
    cache = torch.randn(nb, hkv, bs, 2 * d, generator=g).to(dtype).to(cuda)
    side_k = torch.randn(side, hkv, d, generator=g).to(dtype).to(cuda)
    side_v = torch.randn(side, hkv, d, generator=g).to(dtype).to(cuda)
    kv = N.paged_view(cache, side_k, side_v)
    lib = N.load()
    pages = [5, 0, 36, 37, 38]  # 37: first sidecar page, 38: the partial last one
    pt = torch.tensor(pages, dtype=torch.int64, device=cuda)
    img = torch.full((len(pages), hkv, bs, 2 * d), 7, dtype=dtype, device=cuda)
    st = N.Status(cuda)
    N.check(lib.cs_slide_pack_pages(ctypes.byref(kv), pt.data_ptr(), len(pages),
                                    img.data_ptr(), st.ptr, N.stream_of(cuda)), "pack")
    assert st.read() == 0
    for q, p in enumerate(pages):
        np.testing.assert_array_equal(_bits(img[q]), _bits(_image(cache, side_k, side_v, p, bs)))
    # unpack into a cleared pool: exactly those pages come back
    c2, k2, v2 = torch.zeros_like(cache), torch.zeros_like(side_k), torch.zeros_like(side_v)
    kv2 = N.paged_view(c2, k2, v2)
    N.check(lib.cs_slide_unpack_pages(ctypes.byref(kv2), pt.data_ptr(), len(pages),
                                      img.data_ptr(), st.ptr, N.stream_of(cuda)), "unpack")
    assert st.read() == 0
    for p in (5, 0, 36):
        np.testing.assert_array_equal(_bits(c2[p]), _bits(cache[p]))
    assert int(c2[1].abs().sum()) == 0  # a page not in the list
    np.testing.assert_array_equal(_bits(k2), _bits(side_k))
    np.testing.assert_array_equal(_bits(v2), _bits(side_v))
    # a page outside the arena: status, nothing written
    bad = torch.tensor([39], dtype=torch.int64, device=cuda)
    N.check(lib.cs_slide_pack_pages(ctypes.byref(kv), bad.data_ptr(), 1, img.data_ptr(),
                                    st.ptr, N.stream_of(cuda)), "pack")
    assert st.read() & N.ST_SLOT_RANGE


def test_arena_spill_follows_the_spill_order_and_reloads(cuda):
    arena, key, value, _ = _fixture_arena(cuda)
    arena.write_prefill(key, value)
    sel = torch.tensor([3, 1])
    arena.promote_selected(sel, key[sel] + 1, value[sel] + 2).result()
    key[sel], value[sel] = key[sel] + 1, value[sel] + 2
    n = key.shape[0]
    before = arena.gather(range(n))
    order = arena.spill_order()
    assert order  # some page is eligible
    sp = arena.spill()
    sp.future.result()
    assert sp.pages == order
    view = arena.device_view()
    side_k = arena._side_key if arena._side_key is not None else torch.empty(0)
    side_v = arena._side_value if arena._side_value is not None else torch.empty(0)
    bs = arena.block_size
    for q, p in enumerate(sp.pages):
        want = _image(arena.cache, side_k, side_v, p, bs)
        np.testing.assert_array_equal(_bits(sp.images[q]), _bits(want.cpu()))
    # the pages' records destroyed, then reloaded from the images
    nb = arena.cache.shape[0]
    for p in sp.pages:
        if p < nb:
            arena.cache[p].fill_(-5)
    arena.reload(sp)
    after = arena.gather(range(n))
    assert torch.equal(after[0], before[0]) and torch.equal(after[1], before[1])
    assert view.cache == arena.device_view().cache
    # pins were released: a later write to those tokens is accepted
    arena.update_selected([1, 3], key[[1, 3]] * 2, value[[1, 3]] * 2)
