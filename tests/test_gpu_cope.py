"""CoPE / CCPE attention on the GPU against the reference's golden vectors,
the numpy oracle and the reference's known answers.

Tolerances: float32 inputs vs the float32 reference 1e-4 (summation order);
bf16 inputs 2e-2 abs / 1e-2 rel on the bf16 output;
float64 known answers 1e-9.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import pytest
import torch

from cacheslide_b200.attention import CanonicalPositionPolicy, SelectedAssociationPolicy
from cacheslide_b200.position import (
    CCPEPositionError,
    ChunkResetPositions,
    CoPE,
    cope_attention,
    validate_contextual_path,
)
from oracle import cope as ocope
from tests.conftest import golden

pytestmark = pytest.mark.gpu
G = golden("cope")
F32 = dict(atol=1e-4, rtol=1e-4)
BF16 = dict(atol=2e-2, rtol=1e-2)


def _t(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


def _cope(E, dev, dtype=torch.float32):
    c = CoPE(E.shape[0], E.shape[1], device=dev, dtype=dtype)
    c.position_embeddings.data.copy_(_t(E, dev, dtype))
    return c


def _case(name, dev):
    c = G[name]
    return (_t(c["q"], dev), _t(c["k"], dev), _t(c["v"], dev), _cope(c["E"], dev),
            _t(c["qpos"], dev).long(), c)


def test_plain_matches_golden_with_trace(cuda):
    q, k, v, cope, qpos, c = _case("plain", cuda)
    out, pos = cope_attention(q, k, v, cope, qpos, return_positions=True)
    np.testing.assert_allclose(out.cpu().numpy(), c["out"], **F32)
    np.testing.assert_allclose(pos.cpu().numpy(), c["positions"], atol=1e-4, rtol=1e-5)


def test_decode_and_sparse_keys_match_golden(cuda):
    q, k, v, cope, qpos, c = _case("decode", cuda)
    np.testing.assert_allclose(cope_attention(q, k, v, cope, qpos).cpu().numpy(), c["out"], **F32)
    q, k, v, cope, qpos, c = _case("sparse_keys", cuda)
    out = cope_attention(q, k, v, cope, qpos, _t(c["kpos"], cuda).long())
    np.testing.assert_allclose(out.cpu().numpy(), c["out"], **F32)


def test_association_matches_golden(cuda):
    q, k, v, cope, qpos, c = _case("assoc", cuda)
    policy = SelectedAssociationPolicy(tuple(int(x) for x in c["fixed"]),
                                       _t(c["selected"], cuda).long())
    out = cope_attention(q, k, v, cope, qpos, visibility_transform=policy)
    np.testing.assert_allclose(out.cpu().numpy(), c["out"], **F32)
    # the same policy evaluated as a generic callable (per-chunk mask path)
    out2 = cope_attention(q, k, v, cope, qpos,
                          visibility_transform=lambda a, b: policy(a, b), query_chunk_size=7)
    np.testing.assert_allclose(out2.cpu().numpy(), c["out"], **F32)


def test_masks_match_golden(cuda):
    q, k, v, cope, qpos, c = _case("masks", cuda)
    out = cope_attention(q, k, v, cope, qpos, attention_mask=_t(c["attention_mask"], cuda),
                         visibility_mask=_t(c["visibility_mask"], cuda))
    np.testing.assert_allclose(out.cpu().numpy(), c["out"], **F32)


def test_fixed_positions_match_golden(cuda):
    q, k, v, cope, qpos, c = _case("fixed_positions", cuda)
    out = cope_attention(q, k, v, cope, qpos, fixed_positions=_t(c["positions"], cuda))
    np.testing.assert_allclose(out.cpu().numpy(), c["out"], **F32)


@dataclass(frozen=True)
class _Plan:
    fixed_indices: tuple
    fixed_layout: tuple


class _TableProfile:
    """Profile stand-in with CCPEProfile.lookup's contract (position.py:701-748)."""

    trained_profile_version = "golden-v1"
    chunks = None

    def __init__(self, table, query_positions):
        self.table = torch.from_numpy(table)
        self.known = {int(p): i for i, p in enumerate(query_positions)}

    def lookup(self, chunks, query_positions, key_positions=None, *, checkpoint_id,
               trained_profile_version, strict=True, device=None, dtype=None):
        rows = torch.tensor([self.known[int(p)] for p in query_positions])
        return self.table[:, rows].to(device=device, dtype=dtype)


def _policy(c, mode):
    fixed = tuple(int(x) for x in c["fixed"])
    layout = tuple(("u0", "0" * 64, len(fixed)) for _ in range(1))
    return CanonicalPositionPolicy(_Plan(fixed, layout),
                                   _TableProfile(c["table"], c["table_query_positions"]),
                                   "ck", mode=mode)


def test_canonical_mixed_and_strict_match_golden(cuda):
    q, k, v, cope, qpos, c = _case("canonical_mixed", cuda)
    mixed = _policy(c, "mixed_bias_override")
    out, pos = cope_attention(q, k, v, cope, qpos, positions_transform=mixed,
                              return_positions=True)
    np.testing.assert_allclose(out.cpu().numpy(), c["out"], **F32)
    np.testing.assert_allclose(pos.cpu().numpy(), c["positions"], atol=1e-4, rtol=1e-5)
    with pytest.raises(CCPEPositionError) as err:
        cope_attention(q, k, v, cope, qpos, positions_transform=_policy(c, "strict_contextual"))
    assert str(err.value) == str(c["strict_error"])
    q, k, v, cope, qpos, c = _case("canonical_strict_ok", cuda)
    out = cope_attention(q, k, v, cope, qpos, positions_transform=_policy(c, "strict_contextual"))
    np.testing.assert_allclose(out.cpu().numpy(), c["out"], **F32)


def test_generic_transform_callable_matches_kernel_table_mode(cuda):
    q, k, v, cope, qpos, c = _case("canonical_mixed", cuda)
    pol = _policy(c, "mixed_bias_override")
    out = cope_attention(q, k, v, cope, qpos, positions_transform=lambda p, a, b: pol(p, a, b),
                         query_chunk_size=5)
    np.testing.assert_allclose(out.cpu().numpy(), c["out"], **F32)


def _random(seed, nq, nk, hq, hkv, d, npos, dev, dtype):
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(nk, hq, d, generator=g) / d ** 0.5).to(dtype)
    k = (torch.randn(nk, hkv, d, generator=g) / d ** 0.5).to(dtype)
    v = torch.randn(nk, hkv, d, generator=g).to(dtype)
    E = torch.randn(d, npos, generator=g) * 0.02
    rows = torch.sort(torch.randperm(nk, generator=g)[:nq]).values
    return q[rows], k, v, E, rows


@pytest.mark.parametrize("nk,hq,hkv,d", [(300, 8, 2, 128), (129, 4, 4, 64), (64, 6, 2, 32)])
def test_bf16_gqa_matches_oracle(cuda, nk, hq, hkv, d):
    q, k, v, E, rows = _random(nk, min(nk, 100), nk, hq, hkv, d, 64, cuda, torch.bfloat16)
    want = ocope.cope_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                E.numpy(), rows.numpy())
    got = cope_attention(q.to(cuda), k.to(cuda), v.to(cuda), _cope(E.numpy(), cuda),
                         rows.to(cuda))
    assert got.dtype == torch.bfloat16
    np.testing.assert_allclose(got.float().cpu().numpy(), want, **BF16)


def test_chunk_reset_matches_oracle_and_carry_is_plain(cuda):
    nk, hq, hkv, d, npos = 256, 4, 2, 64, 64
    q, k, v, E, rows = _random(3, 120, nk, hq, hkv, d, npos, cuda, torch.bfloat16)
    key_chunk = torch.arange(nk) // 48
    nch = int(key_chunk.max()) + 1
    g = torch.Generator().manual_seed(5)
    offsets = torch.rand(hq, nk, nch, generator=g) * 30
    offsets[:, :, 1] = -1  # carry through chunk 1
    args = [x.float().numpy() for x in (q, k, v)] + [E.numpy(), rows.numpy()]
    want = ocope.cope_attention(*args, chunk_reset=(key_chunk.numpy(),
                                                    offsets[:, rows].numpy()))
    cope = _cope(E.numpy(), cuda)
    policy = ChunkResetPositions(key_chunk.to(cuda), offsets.to(cuda))
    got = cope_attention(q.to(cuda), k.to(cuda), v.to(cuda), cope, rows.to(cuda),
                         positions_transform=policy)
    np.testing.assert_allclose(got.float().cpu().numpy(), want, **BF16)
    carry = ChunkResetPositions(key_chunk.to(cuda), -torch.ones(hq, nk, nch, device=cuda))
    plain = cope_attention(q.to(cuda), k.to(cuda), v.to(cuda), cope, rows.to(cuda))
    same = cope_attention(q.to(cuda), k.to(cuda), v.to(cuda), cope, rows.to(cuda),
                          positions_transform=carry)
    np.testing.assert_allclose(same.float().cpu().numpy(), plain.float().cpu().numpy(), **BF16)


def test_paged_attention_reads_through_slots(cuda):
    """Attention over a shuffled paged cache equals attention over dense K/V."""
    from cacheslide_b200 import _native as N
    from cacheslide_b200.position import _Holder, _base_params, _launch
    import ctypes  # noqa: F401

    nk, hq, hkv, d, bs = 200, 8, 2, 64, 16
    q, k, v, E, rows = _random(11, 50, nk, hq, hkv, d, 64, cuda, torch.bfloat16)
    q, k, v, rows = q.to(cuda), k.to(cuda), v.to(cuda), rows.to(cuda)
    nb = (nk + bs - 1) // bs + 3
    perm = torch.randperm(nb)[: (nk + bs - 1) // bs]
    cache = torch.zeros(nb, hkv, bs, 2 * d, dtype=torch.bfloat16, device=cuda)
    slots = (perm.to(cuda)[torch.arange(nk, device=cuda) // bs] * bs
             + torch.arange(nk, device=cuda) % bs)
    cache.view(-1, hkv, bs, 2 * d)[slots // bs, :, slots % bs, :d] = k
    cache.view(-1, hkv, bs, 2 * d)[slots // bs, :, slots % bs, d:] = v
    cope = _cope(E.numpy(), cuda)
    dense = cope_attention(q, k, v, cope, rows)
    out = torch.empty_like(dense)
    p = _base_params(q, None, None, _Holder(cope, cope.position_embeddings.detach()),
                     rows, None, nk, hkv, d)
    p.paged = N.paged_view(cache)
    p.kv_slots = slots.data_ptr()
    p.out = out.data_ptr()
    p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
    st = N.Status(cuda)
    p.status = st.ptr
    _launch(p, cuda, allow_fast=False)
    assert st.read() == 0
    np.testing.assert_allclose(out.float().cpu().numpy(), dense.float().cpu().numpy(), **BF16)


@pytest.mark.parametrize("assoc,chunk,paged", [(False, False, False), (True, False, True),
                                               (False, True, True), (True, True, False)])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 1)])
def test_tensor_core_prefill_matches_generic_and_oracle(cuda, assoc, chunk, paged, hq, hkv):
    """cs_cope_attn_prefill (tcgen05) vs cs_cope_attn and the oracle."""
    _tensor_core_case(cuda, assoc, chunk, paged, hq, hkv, 64)


@pytest.mark.parametrize("npos", [96, 128, 101])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 1)])
def test_tensor_core_prefill_wide_position_tables(cuda, npos, hq, hkv):
    """npos 65-128 (the Llama-70B TP8 slice has 128): the q.E table of a row
    is kept in half precision; 101 (not a multiple of 4) takes the element-wise
    E staging."""
    _tensor_core_case(cuda, True, True, True, hq, hkv, npos)


def _tensor_core_case(cuda, assoc, chunk, paged, hq, hkv, npos):
    import ctypes

    from cacheslide_b200 import _native as N
    from cacheslide_b200.position import _Holder, _base_params

    nq, nk, d, bs = 300, 2000, 128, 16
    g = torch.Generator().manual_seed(hq * 7 + assoc + 2 * chunk + 4 * paged + npos)
    q = (torch.randn(nq, hq, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
    k = (torch.randn(nk, hkv, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
    v = torch.randn(nk, hkv, d, generator=g).to(torch.bfloat16).to(cuda)
    rows = torch.sort(torch.randperm(nk, generator=g)[:nq]).values.to(cuda)
    E = torch.randn(d, npos, generator=g) * 0.02
    cope = _cope(E.numpy(), cuda)
    holder = _Holder(cope, cope.position_embeddings.detach())
    fixed = torch.rand(nk, generator=g) < 0.7
    selected = torch.nonzero(fixed & (torch.rand(nk, generator=g) < 0.3)).flatten()
    q_sel = torch.isin(rows.cpu(), selected).to(torch.uint8).to(cuda)
    k_fix = fixed.to(torch.uint8).to(cuda)
    key_chunk = (torch.arange(nk) // 250).to(torch.int32)
    nch = int(key_chunk.max()) + 1
    offsets = torch.rand(hq, nk, nch, generator=g) * 8
    offsets[:, :, 1::3] = -1
    off_rows = offsets[:, rows.cpu()].contiguous().to(cuda)
    kc_dev = key_chunk.to(cuda)
    cache = slots = None
    if paged:
        nb = (nk + bs - 1) // bs + 7
        perm = torch.randperm(nb, generator=g)[: (nk + bs - 1) // bs].to(cuda)
        tok = torch.arange(nk, device=cuda)
        slots = perm[tok // bs] * bs + tok % bs
        cache = torch.zeros(nb, hkv, bs, 2 * d, dtype=torch.bfloat16, device=cuda)
        cache[slots // bs, :, slots % bs, :d] = k
        cache[slots // bs, :, slots % bs, d:] = v
    lib = N.load()
    outs = []
    for fast in (True, False):
        out = torch.empty(nq, hq, d, dtype=torch.bfloat16, device=cuda)
        p = _base_params(q, None if paged else k, None if paged else v, holder, rows, None,
                         nk, hkv, d)
        if paged:
            p.paged = N.paged_view(cache)
            p.kv_slots = slots.data_ptr()
        p.out = out.data_ptr()
        p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
        if assoc:
            p.q_selected, p.k_fixed = q_sel.data_ptr(), k_fix.data_ptr()
        if chunk:
            p.pos_mode = N.POS_CHUNK
            p.key_chunk, p.chunk_off = kc_dev.data_ptr(), off_rows.data_ptr()
            p.co_stride_h, p.co_stride_q = off_rows.stride(0), off_rows.stride(1)
            p.nchunks = nch
        st = N.Status(cuda)
        p.status = st.ptr
        fn = lib.cs_cope_attn_prefill if fast else lib.cs_cope_attn
        N.check(fn(ctypes.byref(p), N.stream_of(cuda)), "prefill" if fast else "generic")
        assert st.read() == 0
        outs.append(out.float().cpu().numpy())
    np.testing.assert_allclose(outs[0], outs[1], **BF16)
    kw = {}
    if assoc:
        kw["visibility_fn"] = lambda a, b: ocope.association_mask(
            a, b, np.nonzero(fixed.numpy())[0], selected.numpy())
    if chunk:
        kw["chunk_reset"] = (key_chunk.numpy(), off_rows.cpu().numpy())
    want = ocope.cope_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                v.float().cpu().numpy(), E.numpy(), rows.cpu().numpy(), **kw)
    np.testing.assert_allclose(outs[0], want, **BF16)


@pytest.mark.parametrize("layout", ["sidecar", "block_major", "dense_strided"])
def test_tensor_core_prefill_copy_paths_agree(cuda, layout, monkeypatch):
    """TMA gather4 and per-row cp.async K/V loads give the generic kernel's result.

    sidecar: 4-key groups wholly in the paged cache, wholly in the sidecar, mixed,
    and one key without a valid slot (zero row, CS_ST_SLOT_RANGE); block_major:
    a [blocks, block_size, heads, 2D] cache seen through a permuted view; and
    dense K/V that are strided views of one fused QKV tensor.
    """
    import ctypes

    from cacheslide_b200 import _native as N
    from cacheslide_b200.position import _Holder, _base_params

    nq, nk, hq, d, bs = 200, 700, 8, 128, 16
    hkv = 1 if layout == "sidecar" else 2  # one head: sidecar rows of a run are consecutive
    g = torch.Generator().manual_seed(41)
    q = (torch.randn(nq, hq, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
    k = (torch.randn(nk, hkv, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
    v = torch.randn(nk, hkv, d, generator=g).to(torch.bfloat16).to(cuda)
    rows = torch.sort(torch.randperm(nk, generator=g)[:nq]).values.to(cuda)
    E = torch.randn(d, 64, generator=g) * 0.02
    cope = _cope(E.numpy(), cuda)
    holder = _Holder(cope, cope.position_embeddings.detach())
    cache = slots = side_k = side_v = None
    kd = vd = None
    expect_status = 0
    tok = torch.arange(nk, device=cuda)
    if layout == "sidecar":
        # 640 native slots: keys 0..599 native, 600..699 in sidecar rows 0..99;
        # in every third 16-key run, keys 2 mod 8 swap sides (native slots
        # 600.., sidecar rows 100..), so there are 16-key runs on both sides and
        # 4-key groups that are all native, all sidecar or mixed
        nb, cap = 40, 200
        slots = tok.clone()
        slots[600:] = nb * bs + torch.arange(nk - 600, device=cuda)
        sw = tok[(tok % 8 == 2) & ((tok // 16) % 3 == 0)]
        slots[sw] = torch.where(sw >= 600, 600 + (sw - 600) // 8, nb * bs + 100 + sw // 8)
        slots[313] = -1
        expect_status = N.ST_SLOT_RANGE
        cache = torch.randn(nb, hkv, bs, 2 * d, generator=g).to(torch.bfloat16).to(cuda)
        side_k = torch.randn(cap, hkv, d, generator=g).to(torch.bfloat16).to(cuda)
        side_v = torch.randn(cap, hkv, d, generator=g).to(torch.bfloat16).to(cuda)
        nat = (slots >= 0) & (slots < nb * bs)
        sn, jn = slots[nat], tok[nat]
        cache[sn // bs, :, sn % bs, :d] = k[jn]
        cache[sn // bs, :, sn % bs, d:] = v[jn]
        sd = (slots >= nb * bs)
        side_k[slots[sd] - nb * bs] = k[tok[sd]]
        side_v[slots[sd] - nb * bs] = v[tok[sd]]
    elif layout == "block_major":
        nb = (nk + bs - 1) // bs + 5
        perm = torch.randperm(nb, generator=g)[: (nk + bs - 1) // bs].to(cuda)
        slots = perm[tok // bs] * bs + tok % bs
        store = torch.zeros(nb, bs, hkv, 2 * d, dtype=torch.bfloat16, device=cuda)
        store[slots // bs, slots % bs, :, :d] = k
        store[slots // bs, slots % bs, :, d:] = v
        cache = store.permute(0, 2, 1, 3)
    else:
        qkv = torch.zeros(nk, 3, hkv, d, dtype=torch.bfloat16, device=cuda)
        qkv[:, 1], qkv[:, 2] = k, v
        kd, vd = qkv[:, 1], qkv[:, 2]
    lib = N.load()
    outs = {}
    for mode in ("tma", "cpasync", "generic"):
        if mode == "cpasync":
            monkeypatch.setenv("CACHESLIDE_PREFILL_COPY", "cpasync")
        else:
            monkeypatch.delenv("CACHESLIDE_PREFILL_COPY", raising=False)
        out = torch.empty(nq, hq, d, dtype=torch.bfloat16, device=cuda)
        p = _base_params(q, kd, vd, holder, rows, None, nk, hkv, d)
        if cache is not None:
            p.paged = N.paged_view(cache, side_k, side_v)
            p.kv_slots = slots.data_ptr()
        p.out = out.data_ptr()
        p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
        st = N.Status(cuda)
        p.status = st.ptr
        fn = lib.cs_cope_attn if mode == "generic" else lib.cs_cope_attn_prefill
        N.check(fn(ctypes.byref(p), N.stream_of(cuda)), mode)
        assert st.read() == expect_status, mode
        outs[mode] = out.float().cpu().numpy()
    np.testing.assert_array_equal(outs["tma"], outs["cpasync"])
    np.testing.assert_allclose(outs["tma"], outs["generic"], **BF16)
    if layout != "sidecar":
        want = ocope.cope_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                    v.float().cpu().numpy(), E.numpy(), rows.cpu().numpy())
        np.testing.assert_allclose(outs["tma"], want, **BF16)


@pytest.mark.parametrize("nk,rows,npos,hq,hkv", [
    (4097, [4096], 64, 32, 8), (1500, [700, 1200, 1499], 64, 32, 8), (513, [512], 64, 32, 8),
    # 71 splits: look-back windows of 32 newer splits, three causal limits
    (9000, [8999, 4500, 100], 64, 32, 8),
    # counts below the last position over most splits: the q.E table path
    (5000, [4999, 2600], 512, 32, 8),
    # one GPU's slice of the Llama-70B TP8 layout: 8 query heads on 1 KV head,
    # npos 128, a 64K context (513 splits)
    (65537, [65536, 30000], 128, 8, 1),
])
def test_split_key_decode_matches_oracle_and_generic(cuda, nk, rows, npos, hq, hkv):
    """Decode rows through the paged cache: split-key kernel vs oracle and vs
    the one-warp-per-row generic kernel."""
    from cacheslide_b200 import _native as N
    from cacheslide_b200.position import _Holder, _base_params

    d, bs = 128, 16
    g = torch.Generator().manual_seed(nk)
    q = (torch.randn(len(rows), hq, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
    k = (torch.randn(nk, hkv, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
    v = torch.randn(nk, hkv, d, generator=g).to(torch.bfloat16).to(cuda)
    E = torch.randn(d, npos, generator=g) * 0.02
    qpos = torch.tensor(rows, device=cuda)
    nb = (nk + bs - 1) // bs + 5
    perm = torch.randperm(nb, generator=g)[: (nk + bs - 1) // bs].to(cuda)
    tok = torch.arange(nk, device=cuda)
    slots = perm[tok // bs] * bs + tok % bs
    cache = torch.zeros(nb, hkv, bs, 2 * d, dtype=torch.bfloat16, device=cuda)
    cache[slots // bs, :, slots % bs, :d] = k
    cache[slots // bs, :, slots % bs, d:] = v
    cope = _cope(E.numpy(), cuda)
    holder = _Holder(cope, cope.position_embeddings.detach())
    outs = []
    lib = N.load()
    for use_decode in (True, False):
        out = torch.empty(len(rows), hq, d, dtype=torch.bfloat16, device=cuda)
        p = _base_params(q, None, None, holder, qpos, None, nk, hkv, d)
        p.paged = N.paged_view(cache)
        p.kv_slots = slots.data_ptr()
        p.out = out.data_ptr()
        p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
        st = N.Status(cuda)
        p.status = st.ptr
        import ctypes

        if use_decode:
            size = lib.cs_cope_attn_decode_workspace(ctypes.byref(p))
            assert size > 0
            ws = torch.empty(size, dtype=torch.uint8, device=cuda)
            N.check(lib.cs_cope_attn_decode(ctypes.byref(p), ws.data_ptr(),
                                            N.stream_of(cuda)), "decode")
        else:
            N.check(lib.cs_cope_attn(ctypes.byref(p), N.stream_of(cuda)), "generic")
        assert st.read() == 0
        outs.append(out.float().cpu().numpy())
    want = ocope.cope_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                v.float().cpu().numpy(), E.numpy(), np.array(rows))
    np.testing.assert_allclose(outs[0], want, **BF16)
    np.testing.assert_allclose(outs[0], outs[1], **BF16)


@pytest.mark.parametrize("hq,hkv,d,npos", [(8, 8, 128, 33), (16, 8, 128, 64), (64, 8, 128, 17),
                                           (32, 8, 64, 64), (12, 4, 96, 40)])
def test_split_key_decode_head_groups_and_widths(cuda, hq, hkv, d, npos):
    """Split-key decode for 1, 2, 4 and 8 query heads per KV head, odd
    position counts, and head widths other than 128 (the general kernels)
    against the oracle."""
    import ctypes

    from cacheslide_b200 import _native as N
    from cacheslide_b200.position import _Holder, _base_params

    nk, bs, rows = 1000, 16, [999, 640]
    g = torch.Generator().manual_seed(hq * 1000 + d + npos)
    q = (torch.randn(len(rows), hq, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
    k = (torch.randn(nk, hkv, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
    v = torch.randn(nk, hkv, d, generator=g).to(torch.bfloat16).to(cuda)
    E = torch.randn(d, npos, generator=g) * 0.05
    nb = (nk + bs - 1) // bs + 3
    perm = torch.randperm(nb, generator=g)[: (nk + bs - 1) // bs].to(cuda)
    tok = torch.arange(nk, device=cuda)
    slots = perm[tok // bs] * bs + tok % bs
    cache = torch.zeros(nb, hkv, bs, 2 * d, dtype=torch.bfloat16, device=cuda)
    cache[slots // bs, :, slots % bs, :d] = k
    cache[slots // bs, :, slots % bs, d:] = v
    cope = _cope(E.numpy(), cuda)
    holder = _Holder(cope, cope.position_embeddings.detach())
    out = torch.empty(len(rows), hq, d, dtype=torch.bfloat16, device=cuda)
    qpos = torch.tensor(rows, device=cuda)  # held: the params keep only its pointer
    p = _base_params(q, None, None, holder, qpos, None, nk, hkv, d)
    p.paged = N.paged_view(cache)
    p.kv_slots = slots.data_ptr()
    p.out = out.data_ptr()
    p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
    st = N.Status(cuda)
    p.status = st.ptr
    lib = N.load()
    size = lib.cs_cope_attn_decode_workspace(ctypes.byref(p))
    assert size > 0
    ws = torch.empty(size, dtype=torch.uint8, device=cuda)
    N.check(lib.cs_cope_attn_decode(ctypes.byref(p), ws.data_ptr(), N.stream_of(cuda)), "decode")
    assert st.read() == 0
    want = ocope.cope_attention(q.float().cpu().numpy(), k.float().cpu().numpy(),
                                v.float().cpu().numpy(), E.numpy(), np.array(rows))
    np.testing.assert_allclose(out.float().cpu().numpy(), want, **BF16)


@pytest.mark.parametrize("layout", ["dense", "paged_sidecar"])
def test_fp16_prefill_and_decode_match_oracle(cuda, layout):
    """float16 inputs through the tensor-core prefill and the tensor-core
    split-key decode (f16 MMA operands), with dense K/V or a paged cache whose
    newest keys live in the sidecar."""
    import ctypes

    from cacheslide_b200 import _native as N
    from cacheslide_b200.position import _Holder, _base_params

    hq, hkv, d, bs, nk = 16, 4, 128, 16, 1100
    g = torch.Generator().manual_seed(97 + (layout == "dense"))
    f16 = torch.float16
    q = (torch.randn(200, hq, d, generator=g) / d ** 0.5).to(f16).to(cuda)
    k = (torch.randn(nk, hkv, d, generator=g) / d ** 0.5).to(f16).to(cuda)
    v = torch.randn(nk, hkv, d, generator=g).to(f16).to(cuda)
    E = torch.randn(d, 64, generator=g) * 0.02
    cope = _cope(E.numpy(), cuda)
    holder = _Holder(cope, cope.position_embeddings.detach())
    pre_rows = torch.sort(torch.randperm(nk, generator=g)[:200]).values.to(cuda)
    dec_rows = torch.tensor([nk - 1, 700], device=cuda)
    cache = slots = side_k = side_v = None
    if layout == "paged_sidecar":
        n_side = 160  # the newest keys are sidecar rows (slots past the native blocks)
        n_native = nk - n_side
        nb = (n_native + bs - 1) // bs + 3
        perm = torch.randperm(nb, generator=g)[: (n_native + bs - 1) // bs].to(cuda)
        tok = torch.arange(n_native, device=cuda)
        native = perm[tok // bs] * bs + tok % bs
        slots = torch.cat([native, nb * bs + torch.arange(n_side, device=cuda)])
        cache = torch.zeros(nb, hkv, bs, 2 * d, dtype=f16, device=cuda)
        cache[native // bs, :, native % bs, :d] = k[:n_native]
        cache[native // bs, :, native % bs, d:] = v[:n_native]
        side_k, side_v = k[n_native:].clone(), v[n_native:].clone()
    lib = N.load()
    keep = []
    for rows, kind in ((pre_rows, "prefill"), (dec_rows, "decode")):
        qq = q[: rows.numel()]
        out = torch.empty(rows.numel(), hq, d, dtype=f16, device=cuda)
        paged = layout != "dense"
        p = _base_params(qq, None if paged else k, None if paged else v, holder, rows, None,
                         nk, hkv, d)
        if paged:
            p.paged = N.paged_view(cache, side_k, side_v)
            p.kv_slots = slots.data_ptr()
        p.out = out.data_ptr()
        p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
        st = N.Status(cuda)
        p.status = st.ptr
        if kind == "prefill":
            N.check(lib.cs_cope_attn_prefill(ctypes.byref(p), N.stream_of(cuda)), kind)
        else:
            size = lib.cs_cope_attn_decode_workspace(ctypes.byref(p))
            ws = torch.empty(size, dtype=torch.uint8, device=cuda)
            keep.append(ws)
            N.check(lib.cs_cope_attn_decode(ctypes.byref(p), ws.data_ptr(), N.stream_of(cuda)),
                    kind)
        assert st.read() == 0, kind
        want = ocope.cope_attention(qq.float().cpu().numpy(), k.float().cpu().numpy(),
                                    v.float().cpu().numpy(), E.numpy(), rows.cpu().numpy())
        np.testing.assert_allclose(out.float().cpu().numpy(), want, **BF16, err_msg=kind)


def test_batched_decode_matches_per_request_decode(cuda):
    """cs_cope_attn_decode_batch over requests of different context lengths
    (and more requests than one launch holds) equals decoding them one by one."""
    import ctypes

    from cacheslide_b200 import _native as N
    from cacheslide_b200.position import _Holder, _base_params

    hq, hkv, d, bs = 32, 8, 128, 16
    lengths = [4097, 130, 1500, 2049, 777, 3000, 64, 900, 4096, 2500]
    g = torch.Generator().manual_seed(5)
    nb = sum((n + bs - 1) // bs for n in lengths) + 4
    cache = torch.zeros(nb, hkv, bs, 2 * d, dtype=torch.bfloat16, device=cuda)
    perm = torch.randperm(nb, generator=g).to(cuda)
    cope = _cope((torch.randn(d, 64, generator=g) * 0.02).numpy(), cuda)
    holder = _Holder(cope, cope.position_embeddings.detach())
    keep, params, singles = [], [], []
    used = 0
    for n in lengths:
        blocks = perm[used:used + (n + bs - 1) // bs]
        used += (n + bs - 1) // bs
        tok = torch.arange(n, device=cuda)
        slots = blocks[tok // bs] * bs + tok % bs
        k = (torch.randn(n, hkv, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
        v = torch.randn(n, hkv, d, generator=g).to(torch.bfloat16).to(cuda)
        cache[slots // bs, :, slots % bs, :d] = k
        cache[slots // bs, :, slots % bs, d:] = v
        q = (torch.randn(1, hq, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
        qpos = torch.tensor([n - 1], device=cuda)
        outs = [torch.empty(1, hq, d, dtype=torch.bfloat16, device=cuda) for _ in range(2)]
        ps = []
        for out in outs:
            p = _base_params(q, None, None, holder, qpos, None, n, hkv, d)
            p.paged = N.paged_view(cache)
            p.kv_slots = slots.data_ptr()
            p.out = out.data_ptr()
            p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
            ps.append(p)
        keep += [slots, q, qpos, *outs]
        params.append(ps[0])
        singles.append((ps[1], outs))
    lib = N.load()
    arr = (N.AttnParams * len(params))(*params)
    size = lib.cs_cope_attn_decode_batch_workspace(arr, len(params))
    assert size > 0
    ws = torch.empty(size, dtype=torch.uint8, device=cuda)
    N.check(lib.cs_cope_attn_decode_batch(arr, len(params), ws.data_ptr(), N.stream_of(cuda)),
            "batch")
    for p, outs in singles:
        wsz = lib.cs_cope_attn_decode_workspace(ctypes.byref(p))
        w1 = torch.empty(wsz, dtype=torch.uint8, device=cuda)
        N.check(lib.cs_cope_attn_decode(ctypes.byref(p), w1.data_ptr(), N.stream_of(cuda)),
                "single")
    torch.cuda.synchronize()
    for _, outs in singles:
        assert torch.equal(outs[0], outs[1])


# ----------------------------------------- reference known answers (float64)
def test_known_visibility_after_gates(cuda):
    cope = CoPE(1, 8, device=cuda, dtype=torch.float64)
    q = torch.ones(1, 1, 1, dtype=torch.float64, device=cuda)
    k = torch.zeros(3, 1, 1, dtype=torch.float64, device=cuda)
    v = torch.tensor([1.0, 10.0, 100.0], dtype=torch.float64, device=cuda)[:, None, None]
    out, trace = cope_attention(q, k, v, cope, torch.tensor([2], device=cuda),
                                visibility_mask=torch.tensor([[True, False, True]], device=cuda),
                                return_positions=True)
    assert out.item() == pytest.approx(50.5, abs=1e-12)
    np.testing.assert_allclose(trace.cpu().numpy(), [[[1.5, 1.0, 0.5]]])


def test_known_association_outputs(cuda):
    policy = SelectedAssociationPolicy((0, 2, 4), torch.tensor([4, 2], device=cuda))
    queries = torch.tensor([4, 1, 2], device=cuda)
    keys = torch.arange(6, device=cuda)
    assert policy(queries, keys).tolist() == [
        [False, True, False, True, True, True],
        [True, True, True, True, True, True],
        [False, True, True, True, False, True],
    ]
    cope = CoPE(1, 16, device=cuda, dtype=torch.float64)
    q = torch.ones(3, 1, 1, dtype=torch.float64, device=cuda)
    k = torch.zeros(6, 1, 1, dtype=torch.float64, device=cuda)
    v = torch.arange(6, dtype=torch.float64, device=cuda)[:, None, None]
    out = cope_attention(q, k, v, cope, queries, visibility_transform=policy)
    np.testing.assert_allclose(out[:, 0, 0].cpu().numpy(), [8 / 3, 0.5, 1.5], atol=1e-12)


def test_known_all_masked_rows_are_zero_and_errors(cuda):
    cope = CoPE(2, 4, device=cuda)
    q, k, v = [torch.ones(2, 1, 2, device=cuda) for _ in range(3)]
    mask = torch.tensor([[False, False], [True, True]], device=cuda)
    out = cope_attention(q, k, v, cope, torch.arange(2, device=cuda), attention_mask=mask)
    assert out[0].abs().sum() == 0 and torch.isfinite(out).all()
    with pytest.raises(ValueError, match="query-dependent"):
        cope_attention(q, k, v, cope, torch.arange(2, device=cuda),
                       fixed_positions=torch.arange(2, device=cuda))
    with pytest.raises(ValueError, match="strictly increasing"):
        cope(q, k, torch.arange(2, device=cuda), torch.tensor([1, 0], device=cuda))
    with pytest.raises(ValueError, match="finite"):
        cope(q * torch.nan, k, torch.arange(2, device=cuda))


def test_known_positions_interpolation_and_validation(cuda):
    cope = CoPE(2, 2, device=cuda)
    logits = torch.zeros(1, 3, 3, device=cuda)
    allowed = torch.ones(3, 3, dtype=torch.bool, device=cuda).tril().unsqueeze(0)
    logits[~allowed] = 1000
    np.testing.assert_allclose(cope.contextual_positions(logits, allowed).cpu().numpy(),
                               [[[0.5, 0, 0], [1, 0.5, 0], [1, 1, 0.5]]])
    c4 = CoPE(1, 4, device=cuda, dtype=torch.float64)
    c4.position_embeddings.data.copy_(torch.tensor([[0, 2, 6, 10]], dtype=torch.float64))
    bias = c4.positional_bias(torch.tensor([[[2.0]]], dtype=torch.float64, device=cuda),
                              torch.tensor([[[0.25, 1.5, 3.0]]], dtype=torch.float64, device=cuda))
    np.testing.assert_allclose(bias.cpu().numpy(), [[[1, 8, 20]]])
    hybrid = torch.tensor([[[1.5, 2, 1.5, 1, 0.5]]], device=cuda)
    with pytest.raises(CCPEPositionError, match="nonincreasing"):
        validate_contextual_path(hybrid, torch.tensor([4], device=cuda),
                                 torch.arange(5, device=cuda))
    with pytest.raises(CCPEPositionError, match="one gate per token"):
        validate_contextual_path(torch.tensor([[[2.75, 0.5]]], device=cuda),
                                 torch.tensor([2], device=cuda), torch.tensor([0, 2], device=cuda))
    validate_contextual_path(torch.tensor([[[2.25, 0.5]]], device=cuda),
                             torch.tensor([2], device=cuda), torch.tensor([0, 2], device=cuda))


def test_future_keys_do_not_change_earlier_rows(cuda):
    g = torch.Generator().manual_seed(8)
    cope = CoPE(2, 6, device=cuda)
    cope.position_embeddings.data.copy_(torch.randn(2, 6, generator=g))
    q, k, v = [torch.randn(4, 2, 2, generator=g).to(cuda) for _ in range(3)]
    original = cope_attention(q, k, v, cope, torch.arange(4, device=cuda))
    k[2:] *= -100
    v[2:] += 100
    changed = cope_attention(q, k, v, cope, torch.arange(4, device=cuda))
    torch.testing.assert_close(changed[:2], original[:2])


@pytest.mark.parametrize("mode", ["high", "low", "carry", "plain"])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 1)])
def test_tensor_core_prefill_skips_inert_tiles_exactly(cuda, mode, hq, hkv):
    """Rows that are all selected (association policy) over a long context of
    mostly fixed keys: the tensor-core kernel takes only the key tiles that
    hold a key some row sees (a non-fixed key or the row's own) or a gate
    that feeds the count of such a key -- the chain from a seen key up to the
    end of the first chunk that restarts the row's count, or up to the row
    itself without restarts.  The result must equal the generic kernel
    (every tile) and the oracle.  Modes: `high` -- every older chunk
    restarts far above npos - 1; `low` -- one chunk restarts low, so the
    gates below its boundary matter; `carry` -- one chunk carries the
    running count instead (offset -1), so a chain crosses its boundary, and
    some rows see keys of their own chunk; `plain` -- contextual positions
    without restarts (every gate from the oldest seen key up is live)."""
    import ctypes

    from cacheslide_b200 import _native as N
    from cacheslide_b200.position import _Holder, _base_params

    nq, nk, d = 64, 4096, 128
    seed = 11 + ["high", "low", "carry", "plain"].index(mode) + 7 * hkv
    g = torch.Generator().manual_seed(seed)
    q = (torch.randn(nq, hq, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
    k = (torch.randn(nk, hkv, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
    v = torch.randn(nk, hkv, d, generator=g).to(torch.bfloat16).to(cuda)
    fixed = torch.ones(nk, dtype=torch.bool)
    fixed[600:610] = False       # a few visible keys far below the rows
    fixed[1800:1830] = False
    if mode in ("carry", "plain"):
        fixed[3300:3306] = False  # seen keys inside the rows' own chunk
    rows = torch.sort(torch.randperm(900, generator=g)[:nq] + 3100).values
    selected = rows.clone()      # every row is a selected (fixed) token
    q_sel = torch.ones(nq, dtype=torch.uint8, device=cuda)
    E = torch.randn(d, 64, generator=g) * 0.02
    cope = _cope(E.numpy(), cuda)
    holder = _Holder(cope, cope.position_embeddings.detach())
    key_chunk = (torch.arange(nk) // 1024).to(torch.int32)
    nch = 4
    offsets = torch.full((hq, nk, nch), 200.0)  # restarts far above npos - 1
    if mode == "low":
        offsets[:, :, 1] = 3.0                  # boundary after key 2047: low restart
    if mode == "carry":
        offsets[:, :, 1] = -1.0                 # chunk 1 carries the running count
    off_rows = offsets[:, rows].contiguous().to(cuda)
    rows_d = rows.to(cuda)
    k_fix = fixed.to(torch.uint8).to(cuda)
    kc_dev = key_chunk.to(cuda)
    chunked = mode != "plain"
    lib = N.load()
    outs = []
    for fast in (True, False):
        out = torch.empty(nq, hq, d, dtype=torch.bfloat16, device=cuda)
        p = _base_params(q, k, v, holder, rows_d, None, nk, hkv, d)
        p.out = out.data_ptr()
        p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
        p.q_selected, p.k_fixed = q_sel.data_ptr(), k_fix.data_ptr()
        if chunked:
            p.pos_mode = N.POS_CHUNK
            p.key_chunk, p.chunk_off = kc_dev.data_ptr(), off_rows.data_ptr()
            p.co_stride_h, p.co_stride_q = off_rows.stride(0), off_rows.stride(1)
            p.nchunks = nch
        st = N.Status(cuda)
        p.status = st.ptr
        fn = lib.cs_cope_attn_prefill if fast else lib.cs_cope_attn
        N.check(fn(ctypes.byref(p), N.stream_of(cuda)), "prefill" if fast else "generic")
        torch.cuda.synchronize(cuda)
        assert st.read() == 0
        outs.append(out.float().cpu().numpy())
    np.testing.assert_allclose(outs[0], outs[1], **BF16)
    kw = {}
    if chunked:
        kw["chunk_reset"] = (key_chunk.numpy(), off_rows.cpu().numpy())
    want = ocope.cope_attention(
        q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), E.numpy(),
        rows.numpy(),
        visibility_fn=lambda a, b: ocope.association_mask(
            a, b, np.nonzero(fixed.numpy())[0], selected.numpy()),
        **kw)
    np.testing.assert_allclose(outs[0], want, **BF16)


def test_batched_prefill_equals_per_request_launches(cuda):
    """cs_cope_attn_prefill_batch (all requests of a step in one grid) gives
    exactly what one cs_cope_attn_prefill launch per request gives, for
    requests of different lengths, positions and association flags."""
    import ctypes

    from cacheslide_b200 import _native as N
    from cacheslide_b200.position import _Holder, _base_params

    d, hq, hkv = 128, 32, 8
    g = torch.Generator().manual_seed(77)
    E = torch.randn(d, 64, generator=g) * 0.02
    cope = _cope(E.numpy(), cuda)
    holder = _Holder(cope, cope.position_embeddings.detach())
    keep, params, outs_b = [], [], []
    for nq, nk in ((40, 300), (300, 1900), (129, 700)):
        q = (torch.randn(nq, hq, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
        k = (torch.randn(nk, hkv, d, generator=g) / d ** 0.5).to(torch.bfloat16).to(cuda)
        v = torch.randn(nk, hkv, d, generator=g).to(torch.bfloat16).to(cuda)
        rows = torch.sort(torch.randperm(nk, generator=g)[:nq]).values.to(cuda)
        fixed = (torch.rand(nk, generator=g) < 0.6).to(torch.uint8).to(cuda)
        qsel = (torch.rand(nq, generator=g) < 0.5).to(torch.uint8).to(cuda)
        out = torch.full((nq, hq, d), float("nan"), dtype=torch.bfloat16, device=cuda)
        p = _base_params(q, k, v, holder, rows, None, nk, hkv, d)
        p.q_selected, p.k_fixed = qsel.data_ptr(), fixed.data_ptr()
        p.out = out.data_ptr()
        p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
        st = N.Status(cuda)
        p.status = st.ptr
        keep.append((q, k, v, rows, fixed, qsel, st))
        params.append(p)
        outs_b.append(out)
    lib = N.load()
    arr = (N.AttnParams * len(params))(*params)
    N.check(lib.cs_cope_attn_prefill_batch(arr, len(params), N.stream_of(cuda)), "batch")
    torch.cuda.synchronize(cuda)
    for p, out_b, kp in zip(params, outs_b, keep):
        assert kp[-1].read() == 0
        single = torch.full_like(out_b, float("nan"))
        p.out = single.data_ptr()
        N.check(lib.cs_cope_attn_prefill(ctypes.byref(p), N.stream_of(cuda)), "single")
        torch.cuda.synchronize(cuda)
        assert torch.equal(single.view(torch.int16), out_b.view(torch.int16))


@pytest.mark.parametrize("case", ["mixed", "strict_valid", "strict_invalid"])
@pytest.mark.parametrize("hq,hkv", [(32, 8), (8, 1)])
def test_tensor_core_table_mode_matches_generic(cuda, case, hq, hkv):
    """Canonical-table mode (CanonicalPositionPolicy, attention.py:32-57) on
    the tensor-core prefill vs the CUDA-core kernel: same outputs and the same
    status bits; strict mode on a table taken from the prompt's own contextual
    positions (a valid path) and on a perturbed table (an invalid one)."""
    import ctypes

    from cacheslide_b200 import _native as N
    from cacheslide_b200.position import _Holder, _base_params

    nq, nk, d, npos = 200, 1500, 128, 64
    g = torch.Generator().manual_seed(hq + len(case))
    q = (torch.randn(nq, hq, d, generator=g) / d ** 0.5).to(torch.bfloat16)
    k = (torch.randn(nk, hkv, d, generator=g) / d ** 0.5).to(torch.bfloat16)
    v = torch.randn(nk, hkv, d, generator=g).to(torch.bfloat16)
    rows = torch.sort(torch.randperm(nk, generator=g)[:nq]).values
    E = torch.randn(d, npos, generator=g) * 0.02
    fixed = torch.sort(torch.randperm(nk, generator=g)[: int(0.7 * nk)]).values
    ordinal = torch.full((nk,), -1, dtype=torch.int32)
    ordinal[fixed] = torch.arange(fixed.numel(), dtype=torch.int32)
    q_row = torch.full((nq,), -1, dtype=torch.int32)
    frows = torch.nonzero(ordinal[rows] >= 0).flatten()
    q_row[frows] = torch.arange(frows.numel(), dtype=torch.int32)
    if case == "mixed":
        table = torch.rand(hq, frows.numel(), fixed.numel(), generator=g) * (npos - 1)
    else:  # the prompt's own (clamped) contextual positions on fixed x fixed
        logits = ocope.qk_logits(q.float().numpy(), k.float().numpy())
        allowed = ocope.causal_mask(rows.numpy(), np.arange(nk))[None].repeat(hq, 0)
        pos = ocope.contextual_positions(logits, allowed, npos)
        table = torch.from_numpy(pos[:, frows.numpy()][:, :, fixed.numpy()].copy())
        if case == "strict_invalid":
            table[:, :, fixed.numel() // 2] += 9.0  # a jump of 9 in one fixed column
            table.clamp_(0, npos - 1)
    dev = lambda t: t.to(cuda)  # noqa: E731
    q, k, v, rows = dev(q), dev(k), dev(v), dev(rows)
    table, q_row_d, k_ord_d = dev(table.float().contiguous()), dev(q_row), dev(ordinal)
    cope = _cope(E.numpy(), cuda)
    holder = _Holder(cope, cope.position_embeddings.detach())
    lib = N.load()
    outs, bits = [], []
    for fast in (True, False):
        out = torch.empty(nq, hq, d, dtype=torch.bfloat16, device=cuda)
        p = _base_params(q, k, v, holder, rows, None, nk, hkv, d)
        p.out = out.data_ptr()
        p.o_stride_tok, p.o_stride_head = out.stride(0), out.stride(1)
        p.pos_mode = N.POS_TABLE
        p.table = table.data_ptr()
        p.tb_stride_h, p.tb_stride_r, p.tb_stride_c = table.stride()
        p.q_row, p.k_ord = q_row_d.data_ptr(), k_ord_d.data_ptr()
        p.strict = 0 if case == "mixed" else 1
        st = N.Status(cuda)
        p.status = st.ptr
        fn = lib.cs_cope_attn_prefill if fast else lib.cs_cope_attn
        N.check(fn(ctypes.byref(p), N.stream_of(cuda)), "prefill" if fast else "generic")
        bits.append(st.read())
        outs.append(out.float().cpu().numpy())
    assert bits[0] == bits[1]
    path_bits = N.ST_PATH_NEG | N.ST_PATH_AVAIL | N.ST_PATH_INCR | N.ST_PATH_GAP
    assert bool(bits[0] & path_bits) == (case == "strict_invalid")
    np.testing.assert_allclose(outs[0], outs[1], **BF16)
