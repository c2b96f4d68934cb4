"""The multi-session chat turn (``chat.ChatTurnStep``, the C4 layout) at a
reduced size (3 sessions at turn 3, messages of 200-400 tokens, 8 decoded
tokens), recomputed on the host from the step's inputs:

* the WCA decisions (``oracle.wca.OracleWCA``: budget, active rows) and the
  fused rows;
* SLIDE relocation is copy-on-write: after the turn the selected history
  rows' canonical slots still hold the snapshot records, their private slots
  the fused rows, the new message's canonical slots its fused (= fresh) rows;
* the attention of the active rows (association policy) and the last decode
  step over the grown context against ``oracle.cope`` (2e-2 / 1e-2).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import cope as ocope
from oracle import wca as owca

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-2, rtol=1e-2)


def _records(cache, slots, bs, d):
    s = slots.to(cache.device)
    rec = cache[s // bs, :, s % bs]
    return rec[..., :d], rec[..., d:]


def test_chat_turn_matches_host_recomputation(cuda):
    from cacheslide_b200.chat import ChatConfig, ChatTurnStep

    cfg = ChatConfig(sessions=3, turn=3, min_tokens=200, max_tokens=400, decode_tokens=8,
                     seed=2)
    step = ChatTurnStep(cfg, cuda)
    host = [dict(ck=s.cached_k.cpu(), cv=s.cached_v.cpu(), calib=s.calib_k.cpu(),
                 fk=s.fresh_k.cpu(), fv=s.fresh_v.cpu(), reused=s.reused.cpu().numpy(),
                 mandatory=s.mandatory.cpu().numpy()) for s in step.sessions]
    stream = torch.cuda.current_stream(cuda).cuda_stream
    step.prefill(stream)
    step.decode(stream)
    torch.cuda.synchronize()
    step.check_status()
    bs, d = cfg.block, cfg.head_dim
    E = step.E.float().cpu().numpy()
    for b, (s, h) in enumerate(zip(step.sessions, host)):
        ck, cv = h["ck"].float().numpy(), h["cv"].float().numpy()
        wca = owca.OracleWCA(correction_fraction=cfg.fraction, epsilon=1e-8, gate_interval=1,
                             convergence_threshold=0.12)
        wca.initialize(ck, h["calib"].float().numpy(), h["reused"], h["mandatory"])
        active = wca.active.copy()
        sel = np.nonzero(wca.selected & ~wca.mandatory)[0]
        assert s.budget == wca.budget
        np.testing.assert_array_equal(s.active.cpu().numpy(), active, err_msg=f"session {b}")
        upd = wca.update(1, ck, cv, h["fk"][active].float().numpy(),
                         h["fv"][active].float().numpy())
        fk = torch.from_numpy(upd["fused_k"]).to(torch.bfloat16)
        fv = torch.from_numpy(upd["fused_v"]).to(torch.bfloat16)
        # copy-on-write relocation
        ok, ov = _records(step.cache, s.canon[torch.from_numpy(sel).to(cuda)], bs, d)
        assert torch.equal(ok.cpu(), h["ck"][sel]) and torch.equal(ov.cpu(), h["cv"][sel])
        pk, pv = _records(step.cache, s.table[torch.from_numpy(active).to(cuda)], bs, d)
        assert torch.equal(pk.cpu().view(torch.int16), fk.view(torch.int16))
        assert torch.equal(pv.cpu().view(torch.int16), fv.view(torch.int16))
        # attention of the active rows over the turn's records
        k, v = h["ck"].clone(), h["cv"].clone()
        k[active], v[active] = fk, fv
        want = ocope.cope_attention(
            s.q.float().cpu().numpy(), k.float().numpy(), v.float().numpy(), E, active,
            visibility_fn=lambda qp, kp: ocope.association_mask(
                qp, kp, np.nonzero(h["reused"])[0], sel))
        np.testing.assert_allclose(s.out.float().cpu().numpy(), want, **TOL,
                                   err_msg=f"session {b}")
        # the last decode step over n + decode_tokens keys
        t = cfg.decode_tokens - 1
        kd = torch.cat([k, s.dec_k.cpu()]).float().numpy()
        vd = torch.cat([v, s.dec_v.cpu()]).float().numpy()
        want = ocope.cope_attention(s.dec_q[t:t + 1].float().cpu().numpy(), kd, vd, E,
                                    np.array([s.n + t]))
        np.testing.assert_allclose(s.dec_out[t:t + 1].float().cpu().numpy(), want, **TOL,
                                   err_msg=f"decode, session {b}")
