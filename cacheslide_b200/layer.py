"""The selective layer loop's QKV projection (runtime.py:409-460 with the
adapter deltas of artifacts.py:189-193) as one tensor-core launch.

At each layer the reference builds the layer's hidden rows for the active
tokens -- rows that were active at the previous layer continue from its
output, rows selected anew are restored from the layer's input snapshot --
with index copies, then runs the QKV projection and the LoRA linears
``F.linear(F.linear(h, qkv_a), qkv_b)`` on them.  ``selective_qkv`` derives
the per-row sources on the device and calls ``cs_qkv_gather_lora``, whose
A-operand load is that gather and whose accumulator also takes the LoRA
delta, so the gathered rows are never materialised.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from . import _native as N


def row_sources(previous: Tensor, active: Tensor, fixed: Tensor, n: int) -> tuple[Tensor, Tensor]:
    """Per active row: 0 and its row in the previous layer's output when it
    was active there, else 1 and its fixed ordinal (its row in the layer's
    snapshot) -- the lookup of runtime.py:416-432.  Raises when a row is in
    neither (the reference's "a mandatory dynamic row was lost")."""
    device = active.device
    lookup = torch.full((n,), -1, dtype=torch.int64, device=device)
    lookup[previous] = torch.arange(previous.numel(), device=device)
    ordinal = torch.full((n,), -1, dtype=torch.int64, device=device)
    ordinal[fixed] = torch.arange(fixed.numel(), device=device)
    rows, restored = lookup[active], ordinal[active]
    continuing = rows >= 0
    if bool(((~continuing) & (restored < 0)).any()):
        raise ValueError("a mandatory dynamic row was lost")
    src = torch.where(continuing, 0, 1).to(torch.int32)
    idx = torch.where(continuing, rows, restored)
    return src.contiguous(), idx.contiguous()


class SelectiveQKV:
    """One layer's prepared launch of ``cs_qkv_gather_lora`` (the arguments of
    ``selective_qkv``, checked and resolved once); ``run(stream)`` enqueues it
    without host synchronisation, ``check()`` reads its status."""

    def __init__(self, previous_hidden: Tensor, previous: Tensor, snapshot_hidden: Tensor,
                 fixed: Tensor, active: Tensor, n: int, weight: Tensor,
                 lora_a: Tensor | None = None, lora_b: Tensor | None = None):
        device = N.require_cuda(weight)
        dt = weight.dtype
        for t in (previous_hidden, snapshot_hidden):
            if t.dtype != dt or t.ndim != 2 or t.shape[1] != weight.shape[1] or \
                    t.stride(1) != 1:
                raise ValueError("hidden rows must be [rows, hidden] with the weight's dtype")
        rank = 0
        if lora_a is not None or lora_b is not None:
            if lora_a is None or lora_b is None:
                raise ValueError("LoRA needs both factors")
            rank = lora_a.shape[0]
            if lora_a.shape[1] != weight.shape[1] or lora_b.shape != (weight.shape[0], rank):
                raise ValueError("LoRA factors must be [rank, hidden] and [n_out, rank]")
            lora_a, lora_b = lora_a.contiguous(), lora_b.contiguous()
        weight = weight.contiguous()
        src, idx = row_sources(previous, active, fixed, n)
        a = active.numel()
        self.device = device
        self.out = torch.empty(a, weight.shape[0], dtype=dt, device=device)
        self.status = N.Status(device)
        self._keep = (previous_hidden, snapshot_hidden, weight, lora_a, lora_b, src, idx)
        p = N.QKVParams()
        p.src0, p.src0_stride, p.src0_rows = (previous_hidden.data_ptr(),
                                              previous_hidden.stride(0), previous_hidden.shape[0])
        p.src1, p.src1_stride, p.src1_rows = (snapshot_hidden.data_ptr(),
                                              snapshot_hidden.stride(0), snapshot_hidden.shape[0])
        p.row_src, p.row_idx, p.a = src.data_ptr(), idx.data_ptr(), a
        p.hidden, p.n_out = weight.shape[1], weight.shape[0]
        p.w = weight.data_ptr()
        p.lora_a = N.ptr(lora_a)
        p.lora_b = N.ptr(lora_b)
        p.rank = rank
        p.out, p.out_stride = self.out.data_ptr(), self.out.stride(0)
        p.dtype = N.DTYPES[dt]
        p.status = self.status.ptr
        self.params = p

    def run(self, stream: int | None = None) -> Tensor:
        s = N.stream_of(self.device) if stream is None else stream
        N.check(N.load().cs_qkv_gather_lora(ctypes.byref(self.params), s), "cs_qkv_gather_lora")
        return self.out

    def check(self) -> None:
        if self.status.read():
            raise ValueError("selective QKV: a row index outside its source, or a timeout")


def selective_qkv(previous_hidden: Tensor, previous: Tensor, snapshot_hidden: Tensor,
                  fixed: Tensor, active: Tensor, n: int, weight: Tensor,
                  lora_a: Tensor | None = None, lora_b: Tensor | None = None) -> Tensor:
    """QKV (+ LoRA delta) of the ``active`` rows of an ``n``-token prompt:
    ``previous_hidden`` holds the previous layer's rows of ``previous``
    (sorted token indices), ``snapshot_hidden`` the layer's input rows of the
    ``fixed`` tokens; ``weight`` is ``[n_out, hidden]``, ``lora_a``
    ``[rank, hidden]``, ``lora_b`` ``[n_out, rank]``.  Returns ``[active,
    n_out]`` in the input dtype (bf16 or fp16)."""
    step = SelectiveQKV(previous_hidden, previous, snapshot_hidden, fixed, active, n, weight,
                        lora_a, lora_b)
    out = step.run()
    step.check()
    return out
