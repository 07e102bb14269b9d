"""Fused elementwise activations restated in NumPy float32 — TEST INFRASTRUCTURE ONLY.

Follows the device helpers and kernel bodies of the reference's fused elementwise kernels
(namitorch/backends/cuda/fused.py:8-69), which agree with its CPU path
(namitorch/_backend.py:124-152 sigmoid / gelu, :156-205 elementwise_forward, :208-222 clamp,
:235-300 derivatives; namitorch/autograd.py:710-771 backward rules):

  sigmoid(x) = 1 / (1 + e) for x >= 0, e / (1 + e) otherwise, e = exp(-|x|)
  silu(x) = x * sigmoid(x), 0 at -inf;  silu'(x) = s + x * s * (1 - s), s where x is not finite
  gelu_tanh(x) = 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), x (or -0) beyond |x| > 20
  gelu_tanh'(x) = 0.5 (1 + t) + 0.5 x (1 - t^2) sqrt(2/pi) (1 + 0.134145 x^2), [x > 0] beyond 20
  relu(x) = max(x, 0) (NaN kept);  relu'(x) = NaN for NaN, else [x > 0]
  clamp: NaN in x or a bound gives x + lo + hi; otherwise x limited to [lo, hi]; its gradient
  passes where lo < x < hi.

`apply(operation, arrays)` takes the seam's operand tuple (see namitorch_b200/backends/fused.py)
and returns the output, or the (first, second) pair for swiglu_backward.
"""
from __future__ import annotations

import numpy as np

F = np.float32
_SCALE = F(0.7978845608028654)
_CUBIC = F(0.044715)
_CUBIC3 = F(0.134145)


def _f(x):
    return np.asarray(x, dtype=np.float32)


def sigmoid(x):
    x = _f(x)
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        e = np.exp(-np.abs(x))
        return np.where(x >= 0, F(1) / (F(1) + e), e / (F(1) + e)).astype(np.float32)


def silu(x):
    x = _f(x)
    with np.errstate(invalid="ignore", over="ignore"):
        return np.where(np.isneginf(x), F(0), x * sigmoid(x)).astype(np.float32)


def silu_grad(x):
    x = _f(x)
    s = sigmoid(x)
    with np.errstate(invalid="ignore", over="ignore", under="ignore"):
        return np.where(np.isfinite(x), s + x * (s * (F(1) - s)), s).astype(np.float32)


def sigmoid_grad(x):
    s = sigmoid(x)
    return (s * (F(1) - s)).astype(np.float32)


def gelu_tanh(x):
    x = _f(x)
    with np.errstate(over="ignore", invalid="ignore", under="ignore"):
        t = np.tanh(_SCALE * (x + _CUBIC * x * x * x))
        inner = (F(0.5) * x) * (F(1) + t)
    outer = np.where(x > 0, x, F(-0.0))
    return np.where(np.abs(x) > 20, outer, inner).astype(np.float32)


def gelu_tanh_grad(x):
    x = _f(x)
    with np.errstate(over="ignore", invalid="ignore", under="ignore"):
        t = np.tanh(_SCALE * (x + _CUBIC * x * x * x))
        d = _SCALE * (F(1) + _CUBIC3 * x * x)
        inner = F(0.5) * (F(1) + t) + F(0.5) * x * (F(1) - t * t) * d
    outer = np.where(x > 0, F(1), F(0))
    return np.where(np.abs(x) > 20, outer, inner).astype(np.float32)


def relu(x):
    x = _f(x)
    return np.where(x <= 0, F(0), x).astype(np.float32)


def relu_grad(x):
    x = _f(x)
    return np.where(np.isnan(x), x, np.where(x > 0, F(1), F(0))).astype(np.float32)


_FORWARD = {"sigmoid": sigmoid, "silu": silu, "gelu_tanh": gelu_tanh, "relu": relu}
_DERIVATIVE = {"sigmoid": sigmoid_grad, "silu": silu_grad, "gelu_tanh": gelu_tanh_grad, "relu": relu_grad}


def _clamp(x, lo, hi, grad=None):
    x = _f(x)
    has_lo, has_hi = lo is not None, hi is not None
    lo = F(0) if lo is None else F(np.asarray(lo, np.float32))
    hi = F(0) if hi is None else F(np.asarray(hi, np.float32))
    with np.errstate(invalid="ignore"):
        bad = np.isnan(x) | np.isnan(lo) | np.isnan(hi)
        nan_out = (x + lo + hi).astype(np.float32)
        if grad is None:
            y = x.copy()
            if has_lo:
                y = np.where(y <= lo, lo, y)
            if has_hi:
                y = np.where(y >= hi, hi, y)
        else:
            inside = np.ones(x.shape, bool)
            if has_lo:
                inside &= x > lo
            if has_hi:
                inside &= x < hi
            y = np.where(inside, _f(grad), F(0))
    return np.where(bad, nan_out, y).astype(np.float32)


def apply(operation: str, arrays):
    """One fused operation on float32 arrays (None for an absent clamp bound)."""
    with np.errstate(over="ignore", invalid="ignore", under="ignore"):
        if operation in ("sigmoid", "silu", "gelu_tanh"):
            return _FORWARD[operation](arrays[0])
        if operation == "sigmoid_backward":
            y, g = _f(arrays[0]), _f(arrays[1])
            return (g * (y * (F(1) - y))).astype(np.float32)
        if operation in ("silu_backward", "gelu_tanh_backward"):
            return (_f(arrays[1]) * _DERIVATIVE[operation[:-9]](arrays[0])).astype(np.float32)
        if operation == "swiglu":
            return (silu(arrays[0]) * _f(arrays[1])).astype(np.float32)
        if operation == "swiglu_backward":
            a, b, g = (_f(x) for x in arrays)
            return ((g * b) * silu_grad(a)).astype(np.float32), (g * silu(a)).astype(np.float32)
        if operation.startswith("bias_"):
            name = operation[5:]
            x = (_f(arrays[0]) + _f(arrays[1])).astype(np.float32)
            if name.endswith("_backward"):
                return (_f(arrays[2]) * _DERIVATIVE[name[:-9]](x)).astype(np.float32)
            return _FORWARD[name](x)
        if operation == "clamp":
            return _clamp(arrays[0], arrays[1], arrays[2])
        if operation == "clamp_backward":
            return _clamp(arrays[0], arrays[1], arrays[2], grad=arrays[3])
    raise ValueError(f"Unsupported fused operation: {operation!r}.")


__all__ = ["apply", "sigmoid", "silu", "silu_grad", "sigmoid_grad", "gelu_tanh", "gelu_tanh_grad", "relu",
           "relu_grad"]
