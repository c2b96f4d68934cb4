"""WCA policy: the seven knobs of Weighted Correction Attention, validated.

The field names, defaults and error messages are the public contract of the
reference's ``WCAConfig`` (``src/cacheslide_vllm/policy.py:21-45``): callers
construct it by keyword and match on the messages.  The validation here is
table driven: ``_RULES`` maps each field to a list of checks, each returning
an error message or ``None``, and the first failing check raises
``ValueError``.

``as_config`` accepts any object that carries the seven attributes -- the
reference's own ``WCAConfig`` included -- and returns a validated
``WCAConfig``, so a caller that still builds the reference's config object
passes it unchanged.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, fields
from typing import Callable, Literal, Optional

Check = Callable[[str, object], Optional[str]]

CONVERGENCE_MODES = ("paper_cosine_lt", "distance_lt")
WEIGHT_UPDATES = ("previous_layer", "same_layer")


def _real(name: str, value: object) -> str | None:
    # bool is a subclass of int; the contract rejects it, and any other type
    # that is not exactly int or float (strings, None, complex, numpy scalars)
    if type(value) is not int and type(value) is not float:
        return f"{name} must be a finite real number, not a boolean"
    try:
        ok = math.isfinite(value)
    except OverflowError:  # an int too large for a float
        ok = False
    return None if ok else f"{name} must be a finite real number"


def _unit_interval(name: str, value: object) -> str | None:
    return None if 0 <= value <= 1 else f"{name} must be in [0, 1]"


def _positive(name: str, value: object) -> str | None:
    return None if value > 0 else f"{name} must be finite and positive"


def _positive_int(name: str, value: object) -> str | None:
    good = type(value) is int and value >= 1
    return None if good else f"{name} must be a positive integer"


def _strict_bool(name: str, value: object) -> str | None:
    return None if type(value) is bool else f"{name} must be a boolean"


def _one_of(options: tuple[str, ...], label: str) -> Check:
    def check(name: str, value: object) -> str | None:
        return None if value in options else f"unknown {label}"

    return check


_RULES: dict[str, list[Check]] = {
    "correction_fraction": [_real, _unit_interval],
    "epsilon": [_real, _positive],
    "convergence_threshold": [_real],
    "gate_interval": [_positive_int],
    "clamp_alpha": [_strict_bool],
    "convergence_mode": [_one_of(CONVERGENCE_MODES, "convergence_mode")],
    "weight_update": [_one_of(WEIGHT_UPDATES, "weight_update")],
}
# numeric fields first, then the rest (the order the contract reports them)
_ORDER = ("correction_fraction", "epsilon", "convergence_threshold", "gate_interval",
          "clamp_alpha", "convergence_mode", "weight_update")


def check_real(name: str, value: object) -> None:
    """Raise ValueError unless ``value`` is a finite int or float (no bool)."""
    message = _real(name, value)
    if message:
        raise ValueError(message)


def validate(values: dict[str, object]) -> None:
    """Run every rule over a field -> value mapping; raise on the first failure.
    The finiteness checks of all numeric fields come before any range check."""
    for name in ("correction_fraction", "epsilon", "convergence_threshold"):
        check_real(name, values[name])
    for name in _ORDER:
        for rule in _RULES[name]:
            if rule is _real:
                continue
            message = rule(name, values[name])
            if message:
                raise ValueError(message)


@dataclass(frozen=True)
class WCAConfig:
    correction_fraction: float = 0.26
    epsilon: float = 1e-8
    gate_interval: int = 4
    convergence_threshold: float = 0.12
    convergence_mode: Literal["paper_cosine_lt", "distance_lt"] = "paper_cosine_lt"
    weight_update: Literal["previous_layer", "same_layer"] = "previous_layer"
    clamp_alpha: bool = False

    def __post_init__(self) -> None:
        validate({f.name: getattr(self, f.name) for f in fields(self)})


FIELDS = tuple(f.name for f in fields(WCAConfig))


def as_config(config: object | None) -> WCAConfig:
    """``None`` -> the defaults; a ``WCAConfig`` as is; any other object with
    the seven attributes (e.g. the reference's config) -> a validated copy."""
    if config is None:
        return WCAConfig()
    if isinstance(config, WCAConfig):
        return config
    missing = [name for name in FIELDS if not hasattr(config, name)]
    if missing:
        raise ValueError(f"WCA config lacks fields: {', '.join(missing)}")
    return WCAConfig(**{name: getattr(config, name) for name in FIELDS})
