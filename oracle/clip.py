"""Total gradient norm and clipping, restated from the reference — TEST INFRASTRUCTURE ONLY.

Follows ``_total_norm`` (namitorch/optim/clip_grad.py:63-79), ``clip_grad_norm_``
(:96-112) and ``clip_grad_value_`` (:115-121) with NumPy arrays standing in for the
gradient tensors.
"""
from __future__ import annotations

import math

import numpy as np


def total_norm(grads: list[np.ndarray], norm_type: float = 2.0) -> np.float64:
    """Two-pass float64 norm: max|g|, then max * (sum (|g|/max)^p)^(1/p)."""
    scale = np.asarray(0.0, dtype=np.float64)
    for g in grads:
        scale = np.maximum(scale, np.max(np.abs(g), initial=0))
    if not bool(np.isfinite(scale)) or bool(scale == 0) or math.isinf(norm_type):
        return np.float64(scale)
    total = np.asarray(0.0, dtype=np.float64)
    with np.errstate(over="ignore", divide="ignore", invalid="ignore", under="ignore"):
        for g in grads:
            scaled = np.abs(np.asarray(g, dtype=np.float64)) / scale
            total = total + np.sum(np.power(scaled, norm_type), dtype=np.float64)
        result = scale * np.power(total, 1 / norm_type)
        if not bool(np.isfinite(result)):
            result = np.exp(np.log(scale) + np.log(total) / norm_type)
    return np.float64(result)


def clip_grad_norm_(grads: list[np.ndarray], max_norm: float, norm_type: float = 2.0,
                    error_if_nonfinite: bool = False, norm: float | None = None) -> np.float64:
    """In-place clip of float arrays; returns the pre-clip norm (float64).

    ``norm``, when given, replaces the computed total norm: a test hands the oracle the norm
    a device reduction produced (equal to the two-pass value to about 1e-15 relative, checked
    separately) so that the clip coefficient, and every value after it, compare bit for bit."""
    norm = total_norm(grads, norm_type) if norm is None else np.float64(norm)
    if error_if_nonfinite and not bool(np.isfinite(norm)):
        raise RuntimeError(f"Cannot clip gradients with nonfinite total norm {norm}.")
    coefficient = np.divide(float(max_norm), np.add(norm, 1e-6))
    if coefficient < 1:
        with np.errstate(invalid="ignore", under="ignore"):
            for g in grads:
                g[...] = np.multiply(np.asarray(g, dtype=np.float64), coefficient).astype(g.dtype)
    return norm


def clip_coefficient(norm: float, max_norm: float) -> float | None:
    """The multiplier clip_grad_norm_ applies, or None when it leaves the gradients alone."""
    coefficient = np.divide(float(max_norm), np.add(np.float64(norm), 1e-6))
    return float(coefficient) if coefficient < 1 else None


def clip_grad_value_(grads: list[np.ndarray], clip_value: float) -> None:
    for g in grads:
        g[...] = np.clip(np.asarray(g, dtype=np.float64), -clip_value, clip_value).astype(g.dtype)
