"""The RAG batch with shared chunks (``rag.RagStep``, the C3 layout) at a
reduced size: the requests' block tables share the pool chunks' blocks, the
turn relocates selected chunk rows copy-on-write (the shared blocks keep the
pool's records), and each request's attention and last decode step match the
host recomputation (``oracle.wca`` decisions and fused rows, ``oracle.cope``
attention with the association policy; 2e-2 / 1e-2)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import cope as ocope
from oracle import wca as owca

pytestmark = pytest.mark.gpu
TOL = dict(atol=2e-2, rtol=1e-2)


def test_rag_batch_matches_host_recomputation(cuda):
    from cacheslide_b200.rag import RagConfig, RagStep

    cfg = RagConfig(requests=4, pool_chunks=6, chunks_per_request=3, chunk_tokens=64,
                    question_tokens=16, decode_tokens=4, seed=3)
    step = RagStep(cfg, cuda)
    assert step.shared_fraction() > 0  # some chunk is read by two requests
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

    def records(slots):
        s = slots.to(cuda)
        rec = step.cache[s // bs, :, s % bs]
        return rec[..., :d].cpu(), rec[..., d:].cpu()

    for b, (s, h) in enumerate(zip(step.sessions, host)):
        # the shared chunk slots still hold the pool's records
        nr = int(h["reused"].sum())
        k0, v0 = records(s.canon[:nr])
        assert torch.equal(k0, h["ck"][:nr]) and torch.equal(v0, h["cv"][:nr])
        ck, cv = h["ck"].float().numpy(), h["cv"].float().numpy()
        wca = owca.OracleWCA(correction_fraction=cfg.fraction, epsilon=1e-8, gate_interval=1,
                             convergence_threshold=0.12)
        wca.initialize(ck, h["calib"].float().numpy(), h["reused"], h["mandatory"])
        active = wca.active.copy()
        sel = np.nonzero(wca.selected & ~wca.mandatory)[0]
        np.testing.assert_array_equal(s.active.cpu().numpy(), active, err_msg=f"request {b}")
        upd = wca.update(1, ck, cv, h["fk"][active].float().numpy(),
                         h["fv"][active].float().numpy())
        fk = torch.from_numpy(upd["fused_k"]).to(torch.bfloat16)
        fv = torch.from_numpy(upd["fused_v"]).to(torch.bfloat16)
        pk, pv = records(s.table[torch.from_numpy(active).to(cuda)])
        assert torch.equal(pk.view(torch.int16), fk.view(torch.int16))
        assert torch.equal(pv.view(torch.int16), fv.view(torch.int16))
        k, v = h["ck"].clone(), h["cv"].clone()
        k[active], v[active] = fk, fv
        want = ocope.cope_attention(
            s.q.float().cpu().numpy(), k.float().numpy(), v.float().numpy(), E, active,
            visibility_fn=lambda qp, kp: ocope.association_mask(
                qp, kp, np.nonzero(h["reused"])[0], sel))
        np.testing.assert_allclose(s.out.float().cpu().numpy(), want, **TOL,
                                   err_msg=f"request {b}")
        t = cfg.decode_tokens - 1
        kd = torch.cat([k, s.dec_k.cpu()]).float().numpy()
        vd = torch.cat([v, s.dec_v.cpu()]).float().numpy()
        want = ocope.cope_attention(s.dec_q[t:t + 1].float().cpu().numpy(), kd, vd, E,
                                    np.array([s.n + t]))
        np.testing.assert_allclose(s.dec_out[t:t + 1].float().cpu().numpy(), want, **TOL,
                                   err_msg=f"decode, request {b}")
