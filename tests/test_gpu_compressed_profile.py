"""Compressed CCPE profiles on the GPU (cs_cope_chunk_offsets through
ChunkResetPositions.from_profile).

* against the reference's calibrated profile (tests/golden/profile.npz): the
  device offsets equal the numpy restatement's, and the attention with them
  reproduces the reference's table-substituted attention
  (CanonicalPositionPolicy, attention.py:32-57) on the calibration's
  representative prompt;
* at the tensor-core kernel's shapes (32 query / 8 KV heads of 128, 1536
  tokens, npos 64): a table calibrated from the prompt itself (its CoPE
  positions on the fixed tokens, as CCPEProfile.calibrate records them) fed
  through the offsets gives the plain CoPE attention of the prompt.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from cacheslide_b200.position import ChunkResetPositions, CoPE, cope_attention
from oracle import cope as oc
from tests.conftest import golden

pytestmark = pytest.mark.gpu
P = golden("profile")


def _t(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


def _cope(E, dev):
    c = CoPE(E.shape[0], E.shape[1], device=dev, dtype=torch.float32)
    c.position_embeddings.data.copy_(_t(E, dev, torch.float32))
    return c


@pytest.mark.parametrize("i", [0, 1, 2])
def test_offsets_match_the_restatement(cuda, i):
    meta, pr = P["meta"], P[f"prompt{i}"]
    n = int(meta["n"])
    q, k = _t(pr["q"], cuda), _t(pr["k"], cuda)
    qpos = torch.arange(n, device=cuda)
    crp = ChunkResetPositions.from_profile(
        _t(meta["table"], cuda), meta["fixed"].tolist(), meta["chunk_lengths"].tolist(), n, q,
        qpos, k, table_query_positions=_t(meta["table_query_positions"], cuda))
    key_seg, soc, last_key, last_ord, ordinal = oc.ccpe_segments(meta["fixed"],
                                                                 meta["chunk_lengths"], n)
    want = oc.chunk_offsets_from_table(pr["q"], pr["k"], np.arange(n), ordinal, key_seg,
                                       last_key, last_ord, soc, meta["table"], n,
                                       int(key_seg.max()) + 1)
    np.testing.assert_array_equal(crp.key_chunk.cpu().numpy(), key_seg)
    np.testing.assert_allclose(crp.offsets.cpu().numpy(), want, atol=2e-6, rtol=0)


def test_attention_reproduces_the_reference_table_policy(cuda):
    meta = P["meta"]
    rep = P[f"prompt{int(meta['representative'])}"]
    n = int(meta["n"])
    q, k, v = _t(rep["q"], cuda), _t(rep["k"], cuda), _t(rep["v"], cuda)
    qpos = torch.arange(n, device=cuda)
    crp = ChunkResetPositions.from_profile(
        _t(meta["table"], cuda), meta["fixed"].tolist(), meta["chunk_lengths"].tolist(), n, q,
        qpos, k, table_query_positions=_t(meta["table_query_positions"], cuda))
    out = cope_attention(q, k, v, _cope(meta["E"], cuda), qpos, positions_transform=crp)
    np.testing.assert_allclose(out.cpu().numpy(), rep["out"], atol=1e-4, rtol=1e-4)


def test_profile_offsets_on_the_tensor_core_path(cuda):
    g = np.random.default_rng(5)
    n, hq, hkv, d, npos = 1536, 32, 8, 128, 64
    lengths = [256, 384, 256, 192]          # fixed chunks
    layout = [("f", 256), ("d", 96), ("f", 384), ("f", 256), ("d", 160), ("f", 192),
              ("d", 192)]
    fixed, t = [], 0
    for kind, length in layout:
        if kind == "f":
            fixed += list(range(t, t + length))
        t += length
    assert t == n and len(fixed) == sum(lengths)
    bf = lambda a: torch.from_numpy(a.astype(np.float32)).to(torch.bfloat16)  # noqa: E731
    q = bf(g.standard_normal((n, hq, d)) / np.sqrt(d))
    k = bf(g.standard_normal((n, hkv, d)) / np.sqrt(d))
    v = bf(g.standard_normal((n, hkv, d)))
    E = (g.standard_normal((d, npos)) * 0.02).astype(np.float32)
    # the calibration record: CoPE positions of the prompt on fixed x fixed
    qf, kf = q.float().numpy(), k.float().numpy()
    logits = oc.qk_logits(qf, kf)
    allowed = oc.causal_mask(np.arange(n), np.arange(n))[None].repeat(hq, 0)
    full = oc.contextual_positions(logits, allowed, npos)
    fx = np.array(fixed)
    table = full[:, fx][:, :, fx]
    rows = np.sort(g.choice(n, 300, replace=False))   # queries: fixed and dynamic rows
    qd = q[rows].to(cuda)
    crp = ChunkResetPositions.from_profile(
        torch.from_numpy(table).to(cuda), fixed, lengths, n, qd,
        torch.from_numpy(rows).to(cuda), k.to(cuda))
    out = cope_attention(qd, k.to(cuda), v.to(cuda), _cope(E, cuda),
                         torch.from_numpy(rows).to(cuda), positions_transform=crp)
    want = oc.cope_attention(qf[rows], kf, v.float().numpy(), E, rows)
    np.testing.assert_allclose(out.float().cpu().numpy(), want, atol=2e-2, rtol=1e-2)
