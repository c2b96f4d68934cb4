"""Layer-pipelined host-to-device snapshot path.

The reference reads each layer's reused K/V snapshot from its page store
(``_prefetch`` submits the next layer's load while the current layer runs,
``_read`` deserialises it, checks shape and finiteness and moves it to the
device with a blocking ``.to(device)``; runtime.py:192-272, storage.py:
453-506).  Here a layer's snapshot arrives from pinned host memory on a copy
stream and lands straight in the layer's paged slots:

* ``SnapshotLoader.submit(layer, key, value, kv, slots)`` enqueues on the
  loader's stream: the H2D copy into a device staging buffer (a ring of
  ``depth`` buffers, so layer L + 1 copies while layer L is scattered and
  computed), a finiteness reduction of the two tensors, and the SLIDE
  scatter into ``slots`` (``cs_slide_scatter``); it returns a ``LayerLoad``.
* ``LayerLoad.wait(stream)`` makes a compute stream wait for the layer (no
  host synchronisation); ``LayerLoad.result()`` waits on the host and raises
  ``ValueError`` when the snapshot held a non-finite value or a slot fell
  outside the arena (the reference's ``_read`` raises for a non-finite
  snapshot).

Staging buffer ``i`` is reused by the load ``depth`` layers later; both run
on the loader's stream, so the reuse is ordered after the earlier scatter.
"""

from __future__ import annotations

import ctypes

import torch

from . import _native as N


class LayerLoad:
    """One submitted layer: its completion event and device flags."""

    def __init__(self, layer: int, event: torch.cuda.Event, finite: torch.Tensor,
                 status: N.Status):
        self.layer = layer
        self.event = event
        self._finite = finite
        self._status = status

    def wait(self, stream: torch.cuda.Stream | None = None) -> None:
        """Make ``stream`` (default: the current one) wait for the layer."""
        (stream or torch.cuda.current_stream(self.event.device)).wait_event(self.event)

    def result(self) -> None:
        """Wait on the host; raise if the snapshot was unusable."""
        self.event.synchronize()
        if not bool(self._finite.item()):
            raise ValueError(f"snapshot tensor is nonfinite at layer {self.layer}")
        bits = self._status.read()
        if bits & N.ST_SLOT_RANGE:
            raise ValueError(f"snapshot slot outside the arena at layer {self.layer}")


class SnapshotLoader:
    """Pinned-memory, layer-pipelined snapshot loads into paged KV slots."""

    def __init__(self, device: torch.device, *, depth: int = 2):
        if type(depth) is not int or depth < 1:
            raise ValueError("depth must be a positive integer")
        N.require_cuda(torch.empty(0, device=device))
        self.device = device
        self.depth = depth
        self.stream = torch.cuda.Stream(device=device)
        self._staging: list[tuple[torch.Tensor, torch.Tensor] | None] = [None] * depth
        self._count = 0

    def _buffers(self, slot: int, shape, dtype) -> tuple[torch.Tensor, torch.Tensor]:
        buf = self._staging[slot]
        if buf is None or buf[0].numel() < shape.numel() or buf[0].dtype != dtype:
            with torch.cuda.stream(self.stream):
                buf = (torch.empty(shape.numel(), dtype=dtype, device=self.device),
                       torch.empty(shape.numel(), dtype=dtype, device=self.device))
            self._staging[slot] = buf
        return buf[0][: shape.numel()].view(shape), buf[1][: shape.numel()].view(shape)

    def submit(self, layer: int, key: torch.Tensor, value: torch.Tensor, kv: N.PagedKV,
               slots: torch.Tensor, *, after: torch.cuda.Event | None = None) -> LayerLoad:
        """Enqueue layer ``layer``'s snapshot: ``key`` / ``value`` are host
        tensors ``[n, kv_heads, head_dim]`` (pinned for an asynchronous
        copy), ``slots`` the device int64 slots of the n tokens in the pool
        ``kv``.  The loader's stream runs independently of the caller's: when
        ``slots`` or the pool were last written (or the pool last read) by
        work on another stream, ``after`` is an event recorded after it."""
        if key.shape != value.shape or key.ndim != 3 or key.dtype != value.dtype:
            raise ValueError("snapshot K and V must share a [n, kv_heads, head_dim] shape")
        if key.device.type != "cpu" or value.device.type != "cpu":
            raise ValueError("snapshots come from host memory")
        if key.dtype not in N.DTYPES or key.dtype != _dtype_of(kv):
            raise ValueError("snapshot dtype differs from the paged cache")
        if (key.shape[1], key.shape[2]) != (kv.kv_heads, kv.head_dim):
            raise ValueError("snapshot tensor geometry is incompatible")
        if slots.dtype != torch.int64 or slots.device != self.device or \
                slots.shape != (key.shape[0],):
            raise ValueError("slots must be a device int64 vector, one per token")
        slot = self._count % self.depth
        self._count += 1
        event = torch.cuda.Event()
        if after is not None:
            self.stream.wait_event(after)
        with torch.cuda.stream(self.stream):
            # flags made on the loader's stream, ordered before their writers
            status = N.Status(self.device)
            finite = torch.empty((), dtype=torch.bool, device=self.device)
            k_dev, v_dev = self._buffers(slot, key.shape, key.dtype)
            k_dev.copy_(key, non_blocking=True)
            v_dev.copy_(value, non_blocking=True)
            torch.logical_and(torch.isfinite(k_dev).all(), torch.isfinite(v_dev).all(),
                              out=finite)
            n = key.shape[0]
            if n:
                N.check(N.load().cs_slide_scatter(
                    ctypes.byref(kv), slots.data_ptr(), None, n, k_dev.data_ptr(),
                    v_dev.data_ptr(), k_dev.stride(0), k_dev.stride(1), status.ptr,
                    self.stream.cuda_stream), "cs_slide_scatter")
            event.record(self.stream)
        # host tensors must outlive the copy: keep them with the load
        load = LayerLoad(layer, event, finite, status)
        load._hold = (key, value, slots)
        return load


def _dtype_of(kv: N.PagedKV) -> torch.dtype:
    for dtype, code in N.DTYPES.items():
        if code == kv.dtype:
            return dtype
    raise ValueError("paged cache dtype is not supported")
