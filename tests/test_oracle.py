"""Pin the numpy oracle: golden vectors made by the reference itself, plus the
reference's own known-answer tests restated (CPU only)."""

from __future__ import annotations

import json

import numpy as np
import pytest

from oracle import cope, slide, wca
from tests.conftest import golden

COPE = golden("cope")
WCA = golden("wca")
PAGED = golden("paged")


def _close(a, b, atol=1e-4, rtol=1e-4):
    """float32 restatement vs float32 reference: only summation order differs."""
    np.testing.assert_allclose(a, b, atol=atol, rtol=rtol)


# ------------------------------------------------------------ golden: CoPE
def test_oracle_plain_and_positions_match_reference():
    c = COPE["plain"]
    out, pos = cope.cope_attention(c["q"], c["k"], c["v"], c["E"], c["qpos"],
                                   return_positions=True)
    _close(out, c["out"])
    _close(pos, c["positions"])


def test_oracle_decode_and_sparse_keys_match_reference():
    c = COPE["decode"]
    _close(cope.cope_attention(c["q"], c["k"], c["v"], c["E"], c["qpos"]), c["out"])
    c = COPE["sparse_keys"]
    _close(cope.cope_attention(c["q"], c["k"], c["v"], c["E"], c["qpos"], c["kpos"]), c["out"])


def test_oracle_association_matches_reference():
    c = COPE["assoc"]
    fn = lambda qp, kp: cope.association_mask(qp, kp, c["fixed"], c["selected"])  # noqa: E731
    _close(cope.cope_attention(c["q"], c["k"], c["v"], c["E"], c["qpos"], visibility_fn=fn),
           c["out"])


def test_oracle_masks_match_reference():
    c = COPE["masks"]
    out = cope.cope_attention(c["q"], c["k"], c["v"], c["E"], c["qpos"],
                              gate_mask=c["attention_mask"], vis_mask=c["visibility_mask"])
    _close(out, c["out"])


def _table_rows(c):
    known = {int(p): i for i, p in enumerate(c["table_query_positions"])}
    return [known[o] for o in range(len(c["fixed"]))]


def test_oracle_canonical_mixed_and_strict_match_reference():
    c = COPE["canonical_mixed"]
    fn = cope.canonical_transform(c["fixed"], c["table"], _table_rows(c))
    out, pos = cope.cope_attention(c["q"], c["k"], c["v"], c["E"], c["qpos"],
                                   positions_fn=fn, return_positions=True)
    _close(out, c["out"])
    _close(pos, c["positions"])
    strict = cope.canonical_transform(c["fixed"], c["table"], _table_rows(c), strict=True)
    with pytest.raises(ValueError) as err:
        cope.cope_attention(c["q"], c["k"], c["v"], c["E"], c["qpos"], positions_fn=strict)
    assert str(err.value) == str(c["strict_error"])
    ok = COPE["canonical_strict_ok"]
    fn = cope.canonical_transform(ok["fixed"], ok["table"], _table_rows(ok), strict=True)
    _close(cope.cope_attention(ok["q"], ok["k"], ok["v"], ok["E"], ok["qpos"], positions_fn=fn),
           ok["out"])


def test_oracle_fixed_positions_match_reference():
    c = COPE["fixed_positions"]
    out = cope.cope_attention(c["q"], c["k"], c["v"], c["E"], c["qpos"],
                              fixed_positions=c["positions"])
    _close(out, c["out"])


def test_chunk_reset_with_carry_offsets_is_plain_cope():
    c = COPE["plain"]
    nk = c["k"].shape[0]
    key_chunk = np.arange(nk) // 16
    offsets = -np.ones((c["q"].shape[1], len(c["qpos"]), key_chunk.max() + 1), np.float32)
    out = cope.cope_attention(c["q"], c["k"], c["v"], c["E"], c["qpos"],
                              chunk_reset=(key_chunk, offsets))
    _close(out, c["out"])
    # exact carries as explicit offsets give the same positions
    logits = cope.qk_logits(c["q"], c["k"])
    allowed = cope.causal_mask(c["qpos"], np.arange(nk))[None]
    gates = np.where(allowed, cope.sigmoid(logits), 0)
    for ch in range(key_chunk.max() + 1):
        end = (ch + 1) * 16
        offsets[:, :, ch] = gates[..., end:].sum(-1)
    _, pos = cope.cope_attention(c["q"], c["k"], c["v"], c["E"], c["qpos"],
                                 chunk_reset=(key_chunk, offsets), return_positions=True)
    _close(pos, c["positions"], atol=2e-5)


# --------------------------------------------- reference known answers (CoPE)
def test_known_gate_reverse_cumsum_clamp():
    # reference tests/test_position.py:16-23
    logits = np.zeros((1, 3, 3), np.float32)
    allowed = np.tril(np.ones((3, 3), bool))[None]
    logits[~allowed] = 1000
    pos = cope.contextual_positions(logits, allowed, 2)
    np.testing.assert_allclose(pos, [[[0.5, 0, 0], [1, 0.5, 0], [1, 1, 0.5]]])


def test_known_interpolation():
    # reference tests/test_position.py:26-35
    E = np.array([[0, 2, 6, 10]], np.float64)
    q = np.array([[[2.0]]])
    bias = cope.positional_bias(q, E, np.array([[[0.25, 1.5, 3.0]]]))
    np.testing.assert_allclose(bias, [[[1, 8, 20]]])


def test_known_visibility_after_gates():
    # reference tests/test_position.py:146-171
    q, k = np.ones((1, 1, 1), np.float32), np.zeros((3, 1, 1), np.float32)
    v = np.array([1.0, 10.0, 100.0], np.float32)[:, None, None]
    E = np.zeros((1, 8), np.float32)
    out, trace = cope.cope_attention(q, k, v, E, np.array([2]),
                                     vis_mask=np.array([[True, False, True]]),
                                     return_positions=True)
    assert out.item() == pytest.approx(50.5)
    np.testing.assert_allclose(trace, [[[1.5, 1.0, 0.5]]])
    _, masked = cope.cope_attention(q, k, v, E, np.array([2]),
                                    gate_mask=np.array([[True, False, True]]),
                                    return_positions=True)
    assert masked[0, 0, 0] == 1


def test_known_hybrid_rejected_and_binade_roundoff_accepted():
    # reference tests/test_position.py:190-237
    hybrid = np.array([[[1.5, 2, 1.5, 1, 0.5]]], np.float32)
    assert cope.validate_contextual_path(hybrid, np.array([4]), np.arange(5)) == \
        cope.NONINCREASING
    assert cope.validate_contextual_path(np.array([[[2.25, 0.5]]], np.float32),
                                         np.array([2]), np.array([0, 2])) is None
    assert cope.validate_contextual_path(np.array([[[2.75, 0.5]]], np.float32),
                                         np.array([2]), np.array([0, 2])) == cope.ONE_GATE
    logits = np.array([100.0] * 128 + [-11.5], np.float32)[None, None]
    pos = cope.contextual_positions(logits, np.ones_like(logits, bool), 256)
    assert (pos[..., :-1] - pos[..., 1:]).max() > 1 + 1e-6
    assert cope.validate_contextual_path(pos, np.array([128]), np.arange(129)) is None


def test_known_association_truth_table_and_outputs():
    # reference tests/test_attention_policies.py:131-153
    queries, keys = np.array([4, 1, 2]), np.arange(6)
    mask = cope.association_mask(queries, keys, (0, 2, 4), [4, 2])
    assert mask.tolist() == [
        [False, True, False, True, True, True],
        [True, True, True, True, True, True],
        [False, True, True, True, False, True],
    ]
    q = np.ones((3, 1, 1))
    k = np.zeros((6, 1, 1))
    v = np.arange(6, dtype=np.float64)[:, None, None]
    fn = lambda qp, kp: cope.association_mask(qp, kp, (0, 2, 4), [4, 2])  # noqa: E731
    out = cope.cope_attention(q, k, v, np.zeros((1, 16)), queries, visibility_fn=fn, chunk=1)
    np.testing.assert_allclose(out[:, 0, 0], [8 / 3, 0.5, 1.5])


# ------------------------------------------------------------- golden: WCA
def test_oracle_wca_sequence_matches_reference():
    s = WCA["sequence"]
    st = wca.OracleWCA(correction_fraction=0.15, gate_interval=2).initialize(
        s["cached"], s["fresh"], s["reused"], s["mandatory"])
    assert st.budget == int(s["budget"])
    np.testing.assert_array_equal(st.initial, s["deviation"])
    np.testing.assert_array_equal(st.active, s["active1"])
    np.testing.assert_allclose(st.alpha, s["alpha0"], rtol=1e-15)
    for layer in (2, 3, 4):
        r = st.update(layer, s[f"L{layer}_ck"], s[f"L{layer}_cv"], s[f"L{layer}_fk"],
                      s[f"L{layer}_fv"])
        np.testing.assert_array_equal(r["indices"], s[f"L{layer}_indices"])
        np.testing.assert_array_equal(r["removed"], s[f"L{layer}_removed"])
        np.testing.assert_array_equal(r["promoted"], s[f"L{layer}_promoted"])
        np.testing.assert_array_equal(r["next_indices"], s[f"L{layer}_next"])
        np.testing.assert_allclose(r["alpha"], s[f"L{layer}_alpha"], rtol=1e-15)
        # the fixture's cache dtype is float32: float64 blend, then one rounding
        np.testing.assert_array_equal(r["fused_k"].astype(np.float32), s[f"L{layer}_fused_k"])
        np.testing.assert_array_equal(r["fused_v"].astype(np.float32), s[f"L{layer}_fused_v"])


def test_oracle_cosine_matches_reference():
    c = WCA["cosine"]
    np.testing.assert_allclose(wca.mean_head_cosine(c["a"], c["b"]), c["cos"], rtol=1e-14)


def test_known_wca_budget_ties_and_weights():
    # reference tests/test_wca.py:23-60
    cached = np.ones((6, 1, 2))
    fresh = np.broadcast_to(np.array([5, 4, 3, 2, 1, 100.0])[:, None, None], cached.shape)
    reused = np.array([True] * 5 + [False])
    st = wca.OracleWCA().initialize(cached, fresh, reused, ~reused)
    assert st.budget == 2
    assert np.nonzero(st.selected)[0].tolist() == [0, 1]
    assert st.active.tolist() == [0, 1, 5]
    tie = np.ones((7, 2, 3))
    mask = np.ones(7, bool)
    assert np.nonzero(wca.OracleWCA().initialize(tie, tie + 1, mask, ~mask).selected)[0].tolist() \
        == [0, 1]
    assert wca.adaptation_weight(np.zeros((1, 1, 2)), np.ones((1, 1, 2)), 0.5).item() == 4
    assert wca.adaptation_weight(np.zeros((1, 1, 2)), np.ones((1, 1, 2)), 0.5, True).item() == 1


def test_select_top_is_stable_descending():
    rng = np.random.default_rng(0)
    keys = rng.integers(0, 20, 500).astype(np.float64)
    avail = rng.random(500) < 0.7
    chosen = wca.select_top(keys, avail, 60)
    order = sorted(np.nonzero(avail)[0], key=lambda i: (-keys[i], i))[:60]
    assert chosen.tolist() == order


# ---------------------------------------------------------- golden: paged
def test_oracle_gather_reproduces_reference_arena_bytes():
    a = PAGED["arena"]
    cache = a["cache"]
    gk, gv = slide.gather(cache, a["side_k"], a["side_v"], a["final_map"][a["order"]])
    np.testing.assert_array_equal(gk, a["gathered_k"])
    np.testing.assert_array_equal(gv, a["gathered_v"])
    stats = json.loads(str(a["stats"]))
    assert stats["physical_hole_reuse"] == 2
