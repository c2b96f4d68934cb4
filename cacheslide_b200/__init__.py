"""cacheslide_b200: CacheSlide's reuse-time attention hot path on B200 (sm_100a).

Modules mirror the reference package ``cacheslide_vllm`` so the path is a
drop-in replacement:

* ``position``  -- ``CoPE``, ``cope_attention``, ``validate_contextual_path``,
  ``CCPEPositionError``, ``ChunkIdentity``, ``ChunkResetPositions``;
* ``attention`` -- ``CanonicalPositionPolicy``, ``SelectedAssociationPolicy``;
* ``wca``       -- ``WCAState``, ``WCAUpdate``, ``squared_deviation``,
  ``adaptation_weight``, ``mean_head_cosine``, ``WCANumericalError``;
* ``policy``    -- ``WCAConfig``;
* ``slide``     -- ``LayerSlotMap``, ``coalesce_slot_writes``, ``SlotWrite``;
* ``paged``     -- ``NativePagedKV``;
* ``errors``    -- ``CacheCapacityError``, ``StaleCompletionError``,
  ``CacheIntegrityError``;
* ``reuse``     -- the fused per-layer reuse-prefill / decode step.

All device arithmetic is in ``_lib/libcacheslide_sm100.so`` (C ABI declared in
``include/cacheslide_b200.h``); build it with ``python -m cacheslide_b200.build``.
"""

__version__ = "0.1.0"
