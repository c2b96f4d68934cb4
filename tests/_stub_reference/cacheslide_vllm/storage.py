"""Storage errors of the stand-in reference package (test fixture)."""


class CacheCapacityError(RuntimeError):
    pass


class CacheIntegrityError(RuntimeError):
    pass


class StaleCompletionError(RuntimeError):
    pass
