"""Stand-in for the reference package in a test: only the module path and the
three storage error classes the runtime catches (names and bases as in the
reference's storage.py:21-31)."""
