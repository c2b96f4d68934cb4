"""WCAConfig validation (the reference's policy contract, policy.py:21-45),
restating the reference's tests/test_wca.py policy cases, plus the adoption of
foreign config objects that carry the same seven fields."""

from __future__ import annotations

from types import SimpleNamespace

import pytest

from cacheslide_b200.policy import WCAConfig, as_config


@pytest.mark.parametrize("field", ["correction_fraction", "epsilon", "convergence_threshold"])
@pytest.mark.parametrize("value", [True, False, "0.26", None, 1j, float("nan"), float("inf"),
                                   10 ** 1000])
def test_numeric_fields_reject_nonfinite_or_non_numeric(field, value):
    with pytest.raises(ValueError, match=field):
        WCAConfig(**{field: value})


@pytest.mark.parametrize("value", [True, False, 4.0, "4", None, 0, -1])
def test_gate_interval_must_be_a_positive_int(value):
    with pytest.raises(ValueError, match="gate_interval"):
        WCAConfig(gate_interval=value)


@pytest.mark.parametrize("value", ["false", "true", 0, 1, None])
def test_clamp_alpha_is_not_truth_coerced(value):
    with pytest.raises(ValueError, match="clamp_alpha"):
        WCAConfig(clamp_alpha=value)


def test_ranges_modes_and_boundaries():
    assert WCAConfig(clamp_alpha=True).clamp_alpha is True
    assert WCAConfig(correction_fraction=0).correction_fraction == 0
    assert WCAConfig(correction_fraction=1, epsilon=1).epsilon == 1
    with pytest.raises(ValueError, match=r"correction_fraction must be in \[0, 1\]"):
        WCAConfig(correction_fraction=1.5)
    with pytest.raises(ValueError, match="epsilon must be finite and positive"):
        WCAConfig(epsilon=0)
    with pytest.raises(ValueError, match="unknown convergence_mode"):
        WCAConfig(convergence_mode="cosine")
    with pytest.raises(ValueError, match="unknown weight_update"):
        WCAConfig(weight_update="next_layer")
    # finiteness of every numeric field is checked before any range
    with pytest.raises(ValueError, match="convergence_threshold must be a finite"):
        WCAConfig(correction_fraction=5, convergence_threshold=float("nan"))


def test_foreign_config_objects_are_adopted_and_validated():
    assert as_config(None) == WCAConfig()
    cfg = WCAConfig(gate_interval=2)
    assert as_config(cfg) is cfg
    fields = dict(correction_fraction=0.15, epsilon=1e-8, gate_interval=3,
                  convergence_threshold=0.2, convergence_mode="distance_lt",
                  weight_update="same_layer", clamp_alpha=True)
    assert as_config(SimpleNamespace(**fields)) == WCAConfig(**fields)
    with pytest.raises(ValueError, match="gate_interval"):
        as_config(SimpleNamespace(**{**fields, "gate_interval": 0}))
    with pytest.raises(ValueError, match="lacks fields: clamp_alpha"):
        as_config(SimpleNamespace(**{k: v for k, v in fields.items() if k != "clamp_alpha"}))
