"""numpy restatement of SLIDE paged KV addressing (TEST INFRASTRUCTURE ONLY).

Follows the reference ``src/cacheslide_vllm/paged.py:205-240`` (slot writes)
and ``paged.py:433-472`` (gather).  The native cache is
``[block, kv_head, block_offset, 2*D]`` with K in ``[..., :D]`` and V in
``[..., D:]``; a slot ``s < blocks*block_size`` addresses
``cache[s // bs, :, s % bs]``, larger slots address the sidecar row
``s - blocks*block_size``.  Arrays are compared as raw integer views, so every
check built on these functions is bit-exact.
"""

from __future__ import annotations

import numpy as np


def split_slots(slots, native_total: int):
    slots = np.asarray(slots, dtype=np.int64)
    native = slots < native_total
    return slots, native


def gather(cache, side_k, side_v, slots):
    """paged.py:433-472 -- K/V rows ``[n, Hkv, D]`` in caller order."""
    nb, hkv, bs, d2 = cache.shape
    d = d2 // 2
    slots, native = split_slots(slots, nb * bs)
    k = np.empty((len(slots), hkv, d), dtype=cache.dtype)
    v = np.empty_like(k)
    s = slots[native]
    k[native] = cache[s // bs, :, s % bs, :d]
    v[native] = cache[s // bs, :, s % bs, d:]
    if (~native).any():
        e = slots[~native] - nb * bs
        k[~native] = side_k[e]
        v[~native] = side_v[e]
    return k, v


def scatter(cache, side_k, side_v, slots, key, value):
    """paged.py:205-240 -- write rows to their native or sidecar slots."""
    nb, hkv, bs, d2 = cache.shape
    d = d2 // 2
    slots, native = split_slots(slots, nb * bs)
    s = slots[native]
    cache[s // bs, :, s % bs, :d] = key[native]
    cache[s // bs, :, s % bs, d:] = value[native]
    if (~native).any():
        e = slots[~native] - nb * bs
        side_k[e] = key[~native]
        side_v[e] = value[~native]


def relocate(cache, side_k, side_v, src_slots, dst_slots):
    """Copy each source slot's K/V record to its destination slot."""
    k, v = gather(cache, side_k, side_v, src_slots)
    scatter(cache, side_k, side_v, dst_slots, k, v)
