"""CPU oracle for the CacheSlide reuse-time hot path (TEST INFRASTRUCTURE ONLY).

This package is a numpy restatement of the reference's arithmetic for the path
the CUDA library implements:

* ``oracle.cope``  -- CoPE/CCPE attention, contextual positions, interpolated
  bias, path validation and the chunk-reset canonical positions
  (reference ``src/cacheslide_vllm/position.py``, ``attention.py``);
* ``oracle.wca``   -- WCA deviation, adaptation weight, mean-head cosine and
  the stable top-budget selection (reference ``src/cacheslide_vllm/wca.py``);
* ``oracle.slide`` -- paged KV slot addressing, gather and scatter
  (reference ``src/cacheslide_vllm/paged.py``).

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` /
``--impl reference`` legs of ``bench.py`` may import it, and only as the checker
or as the timed CPU baseline.  The product (``cacheslide_b200``) never imports
it and has no CPU fallback.

Parity pin: every function here is checked against golden vectors produced by
running the reference itself (``tests/golden/make_golden.py``) and against the
reference's own known-answer tests restated in ``tests/test_oracle.py``.
"""
