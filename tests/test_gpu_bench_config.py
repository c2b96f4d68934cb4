"""Parity at the exact benchmarked configuration (bench.py's default workload).

``reuse.ReuseStep`` over ``SyntheticWorkload(WorkloadConfig())``: 8 requests
of 4096 tokens in 8 chunks of 512 (chunk 3 recomputed), 32 query heads over 8
KV heads of 128, npos 64, paged block 16 with shuffled blocks, WCA 15 %.

Everything the step computes is recomputed on the host from the host copies
of the step's *inputs* (never from what the GPU wrote):

* WCA (wca.py:152-304) by ``oracle.wca.OracleWCA``: the budget, the selected
  and active sets of the calibration layer, then the gated update (cosine
  removal, promotion) and the fused K/V rows, cast to bf16 as torch does;
* the paged cache (paged.py:205-240) by ``oracle.slide``: the baseline
  snapshot written through the request's slot table, then the fused rows over
  it, compared bit-exactly with the device cache read back by plain indexing;
* CCPE attention (position.py:404-560) by ``oracle.cope`` with chunk-reset
  positions and the selected-association policy (attention.py:61-72), on the
  host-built K/V;
* the batched decode over the 4097 keys (the newest token written by the
  step's scatter) against the oracle on the host-built K/V plus that token.

Two requests are checked: the first and the last launched.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import cope as ocope
from oracle import slide as oslide
from oracle import wca as owca

pytestmark = pytest.mark.gpu

TOL = dict(atol=2e-2, rtol=1e-2)  # bf16 inputs, outputs and P


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def _bf16(x: np.ndarray) -> torch.Tensor:
    """float64 -> bf16 exactly as torch's ``.to(torch.bfloat16)`` rounds it
    (the reference's cast of the fused rows, wca.py:262-269)."""
    return torch.from_numpy(x).to(torch.bfloat16)


@pytest.fixture(scope="module")
def bench_step():
    from cacheslide_b200 import reuse

    if not torch.cuda.is_available():
        pytest.fail("GPU test collected on a machine without CUDA")
    cuda = torch.device("cuda:0")

    cfg = reuse.WorkloadConfig()  # the benchmarked defaults
    assert (cfg.requests, cfg.seq, cfg.chunks, cfg.q_heads, cfg.kv_heads) == (8, 4096, 8, 32, 8)
    work = reuse.SyntheticWorkload(cfg, cuda)
    # host copies of the inputs, taken before any kernel has run
    host = []
    for r in work.requests:
        host.append(dict(
            cached_k=r.cached_k.cpu(), cached_v=r.cached_v.cpu(), calib_k=r.calib_k.cpu(),
            fresh_k=r.fresh_k.cpu(), fresh_v=r.fresh_v.cpu(), q_all=r.q_all.cpu(),
            reused=r.reused.cpu().numpy(), mandatory=r.mandatory.cpu().numpy(),
            slots=r.slots_all.cpu().numpy(), key_chunk=r.key_chunk.cpu().numpy(),
            offsets=r.offsets.cpu().numpy(), decode_q=r.decode_q.cpu(),
            decode_k=r.decode_k.cpu(), decode_v=r.decode_v.cpu()))
    step = reuse.ReuseStep(work)
    outs = [o.clone() for o in step.run()]
    torch.cuda.synchronize(cuda)
    step.check_status()
    return cfg, work, step, host, outs


def _host_layer(cfg, h):
    """The whole layer from host inputs: WCA state, fused rows, dense K/V."""
    ck, cv = h["cached_k"].float().numpy(), h["cached_v"].float().numpy()
    wca = owca.OracleWCA(correction_fraction=cfg.fraction, epsilon=1e-8, gate_interval=1,
                         convergence_threshold=0.12)
    wca.initialize(ck, h["calib_k"].float().numpy(), h["reused"], h["mandatory"])
    active = wca.active.copy()
    selected_prev = np.nonzero(wca.selected & ~wca.mandatory)[0]
    upd = wca.update(1, ck, cv, h["fresh_k"][active].float().numpy(),
                     h["fresh_v"][active].float().numpy())
    fk, fv = _bf16(upd["fused_k"]), _bf16(upd["fused_v"])
    # dense K/V of the layer: the snapshot, the fused rows over it
    k, v = h["cached_k"].clone(), h["cached_v"].clone()
    k[active], v[active] = fk, fv
    return wca, active, selected_prev, upd, k, v


@pytest.mark.parametrize("b", [0, 7])
def test_bench_config_step_matches_host_recomputation(bench_step, b):
    cfg, work, step, host, outs = bench_step
    h, r = host[b], work.requests[b]
    wca, active, selected_prev, upd, k, v = _host_layer(cfg, h)

    # WCA decisions: exact index sets
    assert r.budget == wca.budget
    np.testing.assert_array_equal(r.active.cpu().numpy(), active)
    np.testing.assert_array_equal(r.selected_prev.cpu().numpy(), selected_prev)
    np.testing.assert_array_equal(r.selected.cpu().numpy(), wca.selected)
    np.testing.assert_array_equal(r.removed.cpu().numpy(), wca.removed)
    np.testing.assert_array_equal(r.candidate.cpu().numpy(), wca.candidate)
    np.testing.assert_allclose(r.alpha.cpu().numpy(), wca.alpha, rtol=1e-12, atol=0)
    np.testing.assert_allclose(r.used_alpha.cpu().numpy(), upd["alpha"], rtol=1e-12, atol=0)

    # paged cache: snapshot + fused rows, bit-exact through the slot table
    nb, hkv, bs, d2 = work.cache.shape
    cache = np.zeros((nb, hkv, bs, d2), dtype=np.uint16)
    slots = h["slots"][: cfg.seq]
    oslide.scatter(cache, None, None, slots, k.view(torch.int16).numpy().view(np.uint16),
                   v.view(torch.int16).numpy().view(np.uint16))
    s = torch.from_numpy(slots).to(work.cache.device)
    dev_rows = work.cache[s // bs, :, s % bs].cpu().view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(dev_rows, cache[slots // bs, :, slots % bs])

    # CCPE attention of the active rows over the host-built K/V
    want = ocope.cope_attention(
        h["q_all"][active].float().numpy(), k.float().numpy(), v.float().numpy(),
        _np(work.E_acc), active,
        visibility_fn=lambda qp, kp: ocope.association_mask(
            qp, kp, np.nonzero(h["reused"])[0], selected_prev),
        chunk_reset=(h["key_chunk"], h["offsets"][:, active]),
    )
    np.testing.assert_allclose(_np(outs[b]), want, **TOL, err_msg=f"request {b}")


def test_bench_config_decode_matches_host_recomputation(bench_step):
    cfg, work, step, host, _ = bench_step
    dec = [o.clone() for o in step.decode()]
    torch.cuda.synchronize()
    step.check_status()
    n = cfg.seq
    for b in (0, 7):
        h = host[b]
        _, _, _, _, k, v = _host_layer(cfg, h)
        k = torch.cat([k, h["decode_k"]]).float().numpy()
        v = torch.cat([v, h["decode_v"]]).float().numpy()
        want = ocope.cope_attention(h["decode_q"].float().numpy(), k, v, _np(work.E_acc),
                                    np.array([n]))
        np.testing.assert_allclose(_np(dec[b]), want, **TOL, err_msg=f"decode, request {b}")
