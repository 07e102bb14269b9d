"""Option validation and float32 coefficient rounding shared by the optimizers.

Same checks, messages and exception classes as namitorch/optim/_common.py:16-47.
"""
from __future__ import annotations

import math
from numbers import Real

import numpy as np


def _real_option(options: dict, name: str, positive: bool = False, unit_interval: bool = False) -> float:
    """namitorch/optim/_common.py:16-30."""
    if name not in options:
        raise ValueError(f"Missing optimizer option {name!r}.")
    value = options[name]
    if isinstance(value, (bool, np.bool_)) or not isinstance(value, Real):
        raise TypeError(f"Optimizer {name} must be a real scalar.")
    try:
        value = float(value)
    except OverflowError:
        raise ValueError(f"Optimizer {name} must be finite.") from None
    if not math.isfinite(value) or value < 0 or (positive and value == 0) or (unit_interval and value >= 1):
        constraint = "in [0, 1)" if unit_interval else "positive" if positive else "nonnegative"
        raise ValueError(f"Optimizer {name} must be finite and {constraint}.")
    options[name] = value
    return value


def _bool_option(options: dict, name: str) -> bool:
    """namitorch/optim/_common.py:33-36."""
    if name not in options or type(options[name]) is not bool:
        raise TypeError(f"Optimizer {name} must be a Python bool.")
    return options[name]


def _scalar(value: float, name: str = "coefficient") -> np.float32:
    """float64 -> float32 coefficient with the reference's range checks
    (namitorch/optim/_common.py:39-47, float32 parameters)."""
    if not math.isfinite(value) or abs(value) > float(np.finfo(np.float32).max):
        raise ValueError(f"Optimizer {name} must be representable in float32.")
    with np.errstate(under="ignore"):
        result = np.float32(value)
    if name == "eps" and result == 0:
        raise ValueError("Optimizer eps must remain positive in float32.")
    return result
