"""The C5 tensor-parallel step (``tp_step.ShardedReuseStep``) on one GPU, at
a reduced size (2 requests x 4096 tokens, 16 query / 2 KV heads: the C5 head
group of 8 query heads per KV head, npos 128):

* its WCA decisions equal the unsharded ``WCAState``'s on the same inputs
  (one process holds every head: the row sums are complete);
* after a step the paged records hold the snapshot with the fused rows over
  it, and the attention of each request's active rows through those records
  matches the oracle (chunk-reset positions, npos 128, 2e-2 / 1e-2);
* the o_proj rows are the attention rows times the rank's weight block.

The N-rank path (NCCL all-reduces of the row sums and of o_proj) is covered
by ``tests/test_gpu_tp.py`` on 2 GPUs and by ``bench.py`` under torchrun.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import cope as oc

pytestmark = pytest.mark.gpu


def test_tp_step_on_one_gpu(cuda):
    from cacheslide_b200 import _native as N
    from cacheslide_b200.tp_step import ShardedReuseStep, TPWorkloadConfig
    from cacheslide_b200.wca import WCAState

    cfg = TPWorkloadConfig(requests=2, q_heads_total=16, kv_heads_total=2, seq=4096, chunks=8,
                           hidden=512, dynamic_chunk=5)
    step = ShardedReuseStep(cfg, cuda)
    stream = torch.cuda.current_stream(cuda)
    step.run(stream)
    torch.cuda.synchronize()
    step.check_status()
    for b, r in enumerate(step.requests):
        ref = WCAState.initialize(r.cached_k, r.calib_k, r.reused, r.mandatory, step.wca_config)
        assert torch.equal(ref.active_indices, r.active), f"request {b}"
        upd = ref.update(2, r.cached_k, r.cached_v, r.fresh_k[r.active], r.fresh_v[r.active],
                         r.active)
        # the paged records: snapshot with the fused rows over it
        n, hkv, d = cfg.seq, step.hkv, cfg.head_dim
        k = torch.empty(n, hkv, d, dtype=cfg.dtype, device=cuda)
        v = torch.empty_like(k)
        st = torch.zeros(1, dtype=torch.int32, device=cuda)
        N.check(step.lib.cs_slide_gather(ctypes.byref(step.kv), r.slots.data_ptr(), n,
                                         k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1),
                                         st.data_ptr(), N.stream_of(cuda)), "gather")
        torch.cuda.synchronize()
        assert st.item() == 0
        want_k, want_v = r.cached_k.clone(), r.cached_v.clone()
        want_k[r.active], want_v[r.active] = upd.fused_k, upd.fused_v
        assert torch.equal(k.view(torch.int16), want_k.view(torch.int16))
        assert torch.equal(v.view(torch.int16), want_v.view(torch.int16))
        # attention of the active rows
        rows = r.active.cpu().numpy()
        want = oc.cope_attention(
            r.q.float().cpu().numpy(), k.float().cpu().numpy(), v.float().cpu().numpy(),
            step.E.float().cpu().numpy(), rows,
            chunk_reset=(r.key_chunk.cpu().numpy(), r.co.cpu().numpy()))
        np.testing.assert_allclose(r.out.float().cpu().numpy(), want, atol=2e-2, rtol=1e-2,
                                   err_msg=f"request {b}")
        lo, hi = step.row_offsets[b], step.row_offsets[b + 1]
        proj = r.out.view(r.a, -1).float() @ step.w_o.float()
        np.testing.assert_allclose(step.proj[lo:hi].float().cpu().numpy(),
                                   proj.cpu().numpy(), atol=3e-2, rtol=2e-2)
