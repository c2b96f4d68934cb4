"""Exception types shared with the reference runtime's fallback dispatch.

Same class names and bases as ``cacheslide_vllm.storage`` (storage.py:21-31)
so callers that catch them keep working when this package replaces the path.
"""


class CacheCapacityError(RuntimeError):
    """The configured capacity cannot satisfy an operation safely."""


class CacheIntegrityError(RuntimeError):
    """A persisted page failed its identity or checksum check."""


class StaleCompletionError(RuntimeError):
    """An asynchronous operation belongs to a retired store generation."""
