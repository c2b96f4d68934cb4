"""WCA kernels on the GPU against the reference's golden sequence and the oracle.

Index sets (selected / active / removed / promoted, in order) must match
exactly; float64 reductions to ~1e-12 relative (summation order differs);
fused K/V exactly after the cast (float64 blend, one rounding).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from cacheslide_b200 import wca as W
from oracle import wca as owca
from tests.conftest import golden

pytestmark = pytest.mark.gpu


def _t(a, cuda, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(cuda)
    return t if dtype is None else t.to(dtype)


def test_wca_sequence_matches_reference_golden(cuda):
    s = golden("wca")["sequence"]
    cfg = W.WCAConfig(correction_fraction=0.15, gate_interval=2)
    st = W.WCAState.initialize(_t(s["cached"], cuda), _t(s["fresh"], cuda),
                               _t(s["reused"], cuda), _t(s["mandatory"], cuda), cfg)
    assert st.budget == int(s["budget"])
    np.testing.assert_allclose(st.initial_deviation.cpu().numpy(), s["deviation"], rtol=1e-12)
    assert st.active_indices.cpu().tolist() == s["active1"].tolist()
    np.testing.assert_allclose(st.alpha.cpu().numpy(), s["alpha0"], rtol=1e-12)
    for layer in (2, 3, 4):
        r = st.update(layer, _t(s[f"L{layer}_ck"], cuda), _t(s[f"L{layer}_cv"], cuda),
                      _t(s[f"L{layer}_fk"], cuda), _t(s[f"L{layer}_fv"], cuda))
        assert r.indices.cpu().tolist() == s[f"L{layer}_indices"].tolist()
        assert r.removed_indices.cpu().tolist() == s[f"L{layer}_removed"].tolist()
        assert r.promoted_indices.cpu().tolist() == s[f"L{layer}_promoted"].tolist()
        assert r.next_indices.cpu().tolist() == s[f"L{layer}_next"].tolist()
        np.testing.assert_allclose(r.alpha.cpu().numpy(), s[f"L{layer}_alpha"], rtol=1e-12)
        np.testing.assert_array_equal(r.fused_k.cpu().numpy(), s[f"L{layer}_fused_k"])
        np.testing.assert_array_equal(r.fused_v.cpu().numpy(), s[f"L{layer}_fused_v"])


def test_cosine_matches_reference_golden(cuda):
    c = golden("wca")["cosine"]
    got = W.mean_head_cosine(_t(c["a"], cuda), _t(c["b"], cuda)).cpu().numpy()
    np.testing.assert_allclose(got, c["cos"], rtol=1e-13, atol=1e-15)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_cosine_vector_rows_match_oracle(cuda, dtype):
    """16-byte vector path (8 KV heads x 128): mean-head cosine vs the oracle,
    including all-zero heads (cosine 0) and exactly parallel rows."""
    g = torch.Generator().manual_seed(3)
    n, h, d = 257, 8, 128
    a = torch.randn(n, h, d, generator=g).to(dtype)
    b = (a.float() + 0.3 * torch.randn(n, h, d, generator=g)).to(dtype)
    a[5] = 0
    b[6, 3] = 0
    b[7] = a[7]
    got = W.mean_head_cosine(a.to(cuda), b.to(cuda)).cpu().numpy()
    want = owca.mean_head_cosine(a.float().numpy(), b.float().numpy())
    np.testing.assert_allclose(got, want, rtol=1e-13, atol=1e-15)


@pytest.mark.parametrize("n", [1, 33, 4096, 12000, 20000])
def test_select_topk_matches_stable_argsort_with_ties(cuda, n):
    rng = np.random.default_rng(n)
    keys = rng.integers(0, max(2, n // 8), n).astype(np.float64) * 0.25  # many exact ties
    avail = rng.random(n) < 0.8
    slots = max(1, int(0.15 * n))
    expect = owca.select_top(keys, avail, slots)
    sel = torch.zeros(n, dtype=torch.bool, device=cuda)
    chosen = torch.full((slots,), -1, dtype=torch.int64, device=cuda)
    count = torch.zeros(1, dtype=torch.int64, device=cuda)
    from cacheslide_b200 import _native as N

    st = N.Status(cuda)
    keys_d, avail_d = _t(keys, cuda), _t(avail, cuda)  # alive across the launch
    N.check(N.load().cs_wca_select_topk(
        keys_d.data_ptr(), avail_d.data_ptr(), n, slots, sel.data_ptr(),
        chosen.data_ptr(), count.data_ptr(), st.ptr, N.stream_of(cuda)), "select")
    k = int(count.item())
    assert k == len(expect)
    assert chosen[:k].cpu().tolist() == expect.tolist()
    assert sorted(np.nonzero(sel.cpu().numpy())[0].tolist()) == sorted(expect.tolist())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_initialize_update_match_oracle_at_c2_shape(cuda, dtype):
    """C2 shape: n=4096, 8 KV heads x 128, 15% budget, profile K + N(0, 0.05)."""
    g = torch.Generator().manual_seed(7)
    n, h, d = 4096, 8, 128
    cached = (torch.randn(n, h, d, generator=g) / 128 ** 0.5).to(dtype)
    fresh = (cached.float() + 0.05 * torch.randn(n, h, d, generator=g)).to(dtype)
    reused = torch.ones(n, dtype=torch.bool)
    reused[3584:] = False
    mandatory = ~reused
    mandatory[-1] = True
    fresh[~reused] = cached[~reused]
    cfg = W.WCAConfig(correction_fraction=0.15)
    st = W.WCAState.initialize(cached.to(cuda), fresh.to(cuda), reused.to(cuda),
                               mandatory.to(cuda), cfg)
    o = owca.OracleWCA(correction_fraction=0.15).initialize(
        cached.float().numpy(), fresh.float().numpy(), reused.numpy(), mandatory.numpy())
    assert st.budget == o.budget == 538
    assert st.active_indices.cpu().tolist() == o.active.tolist()
    for layer in (2, 3, 4):
        ck = (torch.randn(n, h, d, generator=g) / 128 ** 0.5).to(dtype)
        cv = torch.randn(n, h, d, generator=g).to(dtype)
        rows = torch.from_numpy(o.active)
        fk = (ck[rows].float() + 0.05 * torch.randn(len(rows), h, d, generator=g)).to(dtype)
        fv = (cv[rows].float() + 0.05 * torch.randn(len(rows), h, d, generator=g)).to(dtype)
        r = st.update(layer, ck.to(cuda), cv.to(cuda), fk.to(cuda), fv.to(cuda))
        e = o.update(layer, ck.float().numpy(), cv.float().numpy(), fk.float().numpy(),
                     fv.float().numpy())
        assert r.removed_indices.cpu().tolist() == e["removed"].tolist()
        assert r.promoted_indices.cpu().tolist() == e["promoted"].tolist()
        assert r.next_indices.cpu().tolist() == e["next_indices"].tolist()
        want = torch.from_numpy(e["fused_k"]).to(dtype)
        assert torch.equal(r.fused_k.cpu(), want)


def test_transactional_overflow_leaves_state_untouched(cuda):
    """reference tests/test_wca.py:147-168."""
    half = torch.zeros(1, 1, 1, dtype=torch.float16, device=cuda)
    st = W.WCAState.initialize(half, half + 1, torch.tensor([True], device=cuda),
                               torch.tensor([False], device=cuda))
    before = {k: getattr(st, k).clone() for k in ("alpha", "candidate_mask", "selected_mask",
                                                  "removed_mask")}
    with pytest.raises(W.WCANumericalError, match="overflow"):
        st.update(2, half, half, half + 1, half + 1)
    assert st.last_layer == 1
    for k, v in before.items():
        assert torch.equal(getattr(st, k), v)


def test_weights_and_errors(cuda):
    z = torch.zeros(1, 1, 2, dtype=torch.float16, device=cuda)
    assert W.adaptation_weight(z, torch.ones_like(z), epsilon=0.5).item() == 4
    assert W.adaptation_weight(z, torch.ones_like(z), epsilon=0.5, clamp=True).item() == 1
    zero = torch.zeros(1, 1, 1, dtype=torch.float64, device=cuda)
    with pytest.raises(W.WCANumericalError, match="overflow"):
        W.squared_deviation(zero, zero + 1e308)
    with pytest.raises(W.WCANumericalError, match="finite"):
        W.adaptation_weight(zero + 1, (zero + 1) * torch.nan)
