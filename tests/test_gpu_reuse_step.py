"""The benchmarked step end to end on the GPU (``reuse.ReuseStep``): the
reuse-prefill attention of several requests (SLIDE baseline write, WCA
initialize / select / update / commit, CCPE attention through the paged
slots, each request on its own stream) against the oracle, then the batched
decode of all requests -- one scatter of the newest K/V rows and one
one-pass decode launch -- against the oracle over the n + 1 keys.  The head
shapes are the C2 ones (32 query heads over 8 KV heads of 128), so both the
tensor-core prefill and the one-pass decode kernels run."""

import ctypes

import numpy as np
import pytest
import torch

from oracle import cope as ocope

pytestmark = pytest.mark.gpu

TOL = dict(atol=2e-2, rtol=1e-2)  # bf16 inputs, outputs and P


def test_reuse_step_and_batched_decode_match_oracle(cuda):
    from cacheslide_b200 import _native as N
    from cacheslide_b200 import reuse

    cfg = reuse.WorkloadConfig(requests=3, q_heads=32, kv_heads=8, head_dim=128, seq=1024,
                               chunks=4, npos=64, block=16, fraction=0.15, seed=5)
    work = reuse.SyntheticWorkload(cfg, cuda)
    step = reuse.ReuseStep(work)
    outs = step.run()
    torch.cuda.synchronize()
    step.check_status()
    E = work.E_acc.cpu().numpy()
    for b, r in enumerate(work.requests):
        q, k, v, qpos = reuse.dense_inputs(work, b, step)
        want = ocope.cope_attention(
            q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(), E,
            qpos.cpu().numpy(),
            visibility_fn=lambda a, c, r=r: ocope.association_mask(
                a, c, r.fixed.cpu().numpy(), r.selected_prev.cpu().numpy()),
            chunk_reset=(r.key_chunk.cpu().numpy(), r.offsets[:, qpos.cpu()].cpu().numpy()),
        )
        np.testing.assert_allclose(outs[b].float().cpu().numpy(), want, **TOL,
                                   err_msg=f"request {b}")

    dec = step.decode()
    torch.cuda.synchronize()
    step.check_status()
    n1 = cfg.seq + 1
    for b, r in enumerate(work.requests):
        k = torch.empty(n1, cfg.kv_heads, cfg.head_dim, dtype=cfg.dtype, device=cuda)
        v = torch.empty_like(k)
        st = torch.zeros(1, dtype=torch.int32, device=cuda)
        N.check(step.lib.cs_slide_gather(
            ctypes.byref(step.kv), r.dec_slots.data_ptr(), n1, k.data_ptr(), v.data_ptr(),
            k.stride(0), k.stride(1), st.data_ptr(), N.stream_of(cuda)), "gather")
        torch.cuda.synchronize()
        assert st.item() == 0
        want = ocope.cope_attention(
            r.decode_q.float().cpu().numpy(), k.float().cpu().numpy(),
            v.float().cpu().numpy(), E, r.dec_pos.cpu().numpy())
        np.testing.assert_allclose(dec[b].float().cpu().numpy(), want, **TOL,
                                   err_msg=f"decode, request {b}")
