"""Decode through the allocation-free entry point (cs_cope_attn_decode_noalloc).

Callers such as a plugin inside an inference engine, which has already given
all free HBM to its KV-cache pool, or a foreign-language host without a CUDA
allocator, cannot allocate the decode workspace.  This entry point takes its
scratch from static device memory inside the library.  The test calls it
through the C ABI and checks it against cs_cope_attn_decode (workspace
supplied by the caller) on two calls in a row, with different inputs, since
every call reuses the same static array.  It lives in its own file, collected
after all other tests, and passes alone in a fresh process as well.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from cacheslide_b200 import _native as N
from cacheslide_b200.position import CoPE, _base_params, _Holder

pytestmark = pytest.mark.gpu
BF16 = dict(atol=2e-2, rtol=1e-2)  # the tolerance of the other bf16 attention tests


def _problem(dev, seed, nk, rows):
    hq, hkv, d, bs = 32, 8, 128, 16
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(len(rows), hq, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(dev)
    k = (torch.randn(nk, hkv, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(dev)
    v = torch.randn(nk, hkv, d, generator=g).to(torch.bfloat16).to(dev)
    nb = (nk + bs - 1) // bs + 3
    perm = torch.randperm(nb, generator=g)[: (nk + bs - 1) // bs].to(dev)
    tok = torch.arange(nk, device=dev)
    slots = perm[tok // bs] * bs + tok % bs
    cache = torch.zeros(nb, hkv, bs, 2 * d, dtype=torch.bfloat16, device=dev)
    cache[slots // bs, :, slots % bs, :d] = k
    cache[slots // bs, :, slots % bs, d:] = v
    cope = CoPE(d, 64, device=dev)
    cope.position_embeddings.data.copy_((torch.randn(d, 64, generator=g) * 0.02).to(dev))
    qpos = torch.tensor(rows, device=dev)
    keep = (q, cache, slots, qpos, cope)
    return keep


def _params(keep, out):
    q, cache, slots, qpos, cope = keep
    p = _base_params(q, None, None, _Holder(cope, cope.position_embeddings.detach()), qpos, None,
                     slots.numel(), cache.shape[1], cache.shape[3] // 2)
    p.paged = N.paged_view(cache)
    p.kv_slots = slots.data_ptr()
    p.out = out.data_ptr()
    p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
    return p


def _run(keep, noalloc: bool) -> np.ndarray:
    q = keep[0]
    dev = q.device
    lib = N.load()
    out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16, device=dev)
    p = _params(keep, out)
    st = N.Status(dev)
    p.status = st.ptr
    if noalloc:
        rc = lib.cs_cope_attn_decode_noalloc(ctypes.byref(p), N.stream_of(dev))
    else:
        size = lib.cs_cope_attn_decode_workspace(ctypes.byref(p))
        ws = torch.empty(size, dtype=torch.uint8, device=dev)
        rc = lib.cs_cope_attn_decode(ctypes.byref(p), ws.data_ptr(), N.stream_of(dev))
    assert rc == N.CS_OK
    torch.cuda.synchronize(dev)
    assert st.read() == 0
    return out.float().cpu().numpy()


def test_noalloc_decode_matches_workspace_decode_on_two_calls(cuda):
    first = _problem(cuda, 1, 4097, [4096])
    second = _problem(cuda, 2, 1500, [700, 1200, 1499])
    for keep in (first, second):
        got = _run(keep, noalloc=True)
        want = _run(keep, noalloc=False)
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, want, **BF16)


def test_noalloc_decode_calls_queued_back_to_back_on_one_stream(cuda):
    # the supported way to share the array: stream-ordered calls, one sync
    probs = [_problem(cuda, 4, 2500, [2499]), _problem(cuda, 5, 900, [300, 899])]
    lib = N.load()
    outs, holds = [], []
    for keep in probs:
        q = keep[0]
        out = torch.full(q.shape, float("nan"), dtype=torch.bfloat16, device=cuda)
        p = _params(keep, out)
        st = N.Status(cuda)
        p.status = st.ptr
        assert lib.cs_cope_attn_decode_noalloc(ctypes.byref(p), N.stream_of(cuda)) == N.CS_OK
        outs.append(out)
        holds.append((p, st))
    torch.cuda.synchronize(cuda)
    for (_, st), out, keep in zip(holds, outs, probs):
        assert st.read() == 0
        got = out.float().cpu().numpy()
        assert np.isfinite(got).all()
        np.testing.assert_allclose(got, _run(keep, noalloc=False), **BF16)


def test_noalloc_decode_rejects_problems_beyond_the_static_capacity(cuda):
    keep = _problem(cuda, 3, 33000, [32999] * 1 + [32998])  # ~9 MB per row pair
    q = keep[0]
    big_rows = torch.arange(32000, 32016, device=cuda)  # 16 rows x 32 heads x 33000 keys
    keep = (q.new_zeros(16, q.shape[1], q.shape[2]), keep[1], keep[2], big_rows, keep[4])
    out = torch.empty(16, q.shape[1], q.shape[2], dtype=torch.bfloat16, device=cuda)
    p = _params(keep, out)
    lib = N.load()
    assert lib.cs_cope_attn_decode_workspace(ctypes.byref(p)) > (16 << 20)
    assert lib.cs_cope_attn_decode_noalloc(ctypes.byref(p), N.stream_of(cuda)) == \
        N.CS_ERR_TOO_LARGE
