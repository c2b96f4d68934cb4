"""Compressed CCPE profiles: the reference's canonical tables (CCPEProfile,
position.py:581-748, applied by CanonicalPositionPolicy, attention.py:32-57)
turned into per-chunk carried counts for the chunk-reset positions of the
attention kernels (cs_cope_chunk_offsets).

The fixture (tests/golden/profile.npz, made by make_golden.py from the
reference) holds a profile calibrated from three prompts that share their
fixed chunks and differ in their dynamic tokens, and the reference's
table-substituted attention on each prompt.  On CPU the numpy restatement is
checked against it:

* on the calibration's representative prompt the chunk-reset positions equal
  the reference's table-substituted positions in every cell, and the
  attention outputs agree;
* on the other prompts every fixed x fixed cell equals its table entry (the
  dynamic cells follow the chunk-reset carry, not the reference's current
  contextual count: the compressed form keeps the table only for fixed keys).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import cope as oc

GOLD = np.load(Path(__file__).resolve().parent / "golden" / "profile.npz")


def _case(name):
    pre = name + "__"
    return {k[len(pre):]: GOLD[k] for k in GOLD.files if k.startswith(pre)}


META = _case("meta")


def _compressed(prompt):
    n = int(META["n"])
    fixed, lengths = META["fixed"], META["chunk_lengths"]
    key_seg, seg_of_chunk, last_key, last_ord, ordinal = oc.ccpe_segments(fixed, lengths, n)
    rows = {int(o): i for i, o in enumerate(META["table_query_positions"])}
    q_ord = np.array([rows[o] if o >= 0 else -1 for o in ordinal])
    qpos = np.arange(n)
    offsets = oc.chunk_offsets_from_table(
        prompt["q"], prompt["k"], qpos, q_ord, key_seg[qpos], last_key, last_ord,
        seg_of_chunk, META["table"], n, int(key_seg.max()) + 1)
    return key_seg, offsets


def _positions(prompt, key_seg, offsets):
    q, k = prompt["q"], prompt["k"]
    n = q.shape[0]
    logits = oc.qk_logits(q, k)
    allowed = oc.causal_mask(np.arange(n), np.arange(n))[None].repeat(q.shape[1], 0)
    npos = META["E"].shape[1]
    return oc.chunk_reset_positions(logits, allowed, key_seg, offsets, key_seg, npos)


def test_segments_follow_the_fixed_layout():
    key_seg, soc, last_key, last_ord, ordinal = oc.ccpe_segments(
        [0, 1, 2, 5, 6, 7, 8, 10, 11], [3, 4, 2], 13)
    assert key_seg.tolist() == [0, 0, 0, 1, 1, 2, 2, 2, 2, 3, 4, 4, 5]
    assert soc.tolist() == [0, 2, 4] and last_key.tolist() == [2, 8, 11]
    assert last_ord.tolist() == [2, 6, 8]
    assert ordinal.tolist() == [0, 1, 2, -1, -1, 3, 4, 5, 6, -1, 7, 8, -1]


def test_representative_prompt_reproduces_the_table_everywhere():
    rep = _case(f"prompt{int(META['representative'])}")
    key_seg, offsets = _compressed(rep)
    got = _positions(rep, key_seg, offsets)
    np.testing.assert_allclose(got, rep["positions"], atol=1e-5, rtol=0)
    out = oc.cope_attention(rep["q"], rep["k"], rep["v"], META["E"], np.arange(rep["q"].shape[0]),
                            chunk_reset=(key_seg, offsets))
    np.testing.assert_allclose(out, rep["out"], atol=1e-5, rtol=1e-5)


@pytest.mark.parametrize("i", [0, 1, 2])
def test_fixed_cells_equal_the_table_on_every_prompt(i):
    prompt = _case(f"prompt{i}")
    key_seg, offsets = _compressed(prompt)
    got = _positions(prompt, key_seg, offsets)
    fixed = META["fixed"]
    cells = np.ix_(np.arange(got.shape[0]), fixed, fixed)
    np.testing.assert_allclose(got[cells], prompt["positions"][cells], atol=1e-5, rtol=0)
    # the table itself, for the fixed rows and columns (causal cells)
    table = META["table"]
    causal = fixed[None, :] <= fixed[:, None]
    np.testing.assert_allclose(np.where(causal, got[cells], 0),
                               np.where(causal, table, 0), atol=1e-5, rtol=0)
