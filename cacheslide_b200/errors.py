"""Exception types shared with the reference runtime's fallback dispatch.

The reference runtime catches ``cacheslide_vllm.storage.CacheCapacityError``
(and the other two storage errors) to fall back to a full prefill.  When the
reference package is importable in the same process -- the drop-in setting,
where its runtime drives these operators -- this module re-exports those very
classes, so the runtime's ``except`` clauses catch what the slot map and the
paged arena raise without any edit.  Otherwise it defines classes of the same
names and bases (``RuntimeError``, as in storage.py:21-31).
"""

from __future__ import annotations

try:  # the reference's own classes, when its package is installed
    from cacheslide_vllm.storage import (  # type: ignore[import-not-found]
        CacheCapacityError,
        CacheIntegrityError,
        StaleCompletionError,
    )

    SHARED_WITH_REFERENCE = True
except ImportError:
    SHARED_WITH_REFERENCE = False

    class CacheCapacityError(RuntimeError):  # type: ignore[no-redef]
        """The configured capacity cannot satisfy an operation safely."""

    class CacheIntegrityError(RuntimeError):  # type: ignore[no-redef]
        """A persisted page failed its identity or checksum check."""

    class StaleCompletionError(RuntimeError):  # type: ignore[no-redef]
        """An asynchronous operation belongs to a retired store generation."""


__all__ = ["CacheCapacityError", "CacheIntegrityError", "StaleCompletionError",
           "SHARED_WITH_REFERENCE"]
