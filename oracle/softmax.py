"""Row softmax family restated in NumPy float32 — TEST INFRASTRUCTURE ONLY.

Follows the reference's fused row-softmax kernels (namitorch/backends/cuda/softmax.py:41-88)
and their host checks (:91-178): softmax over the last dimension of the allowed entries,
allowed = causal rule (column <= min(offset, width) + row % queries) and a boolean mask
broadcast over rows (``mask_rows``, :91-107); an empty row (no allowed finite value) gives
zeros, a row whose max is NaN or +inf gives NaN; backward y * (g - sum(g * y)) on the
allowed entries, 0 elsewhere. The same arithmetic as the reference's CPU path where both
apply (namitorch/_backend.py:321-354, namitorch/autograd.py:538-564).
"""
from __future__ import annotations

import numpy as np


def mask_rows(mask_shape, shape):
    """namitorch/backends/cuda/softmax.py:91-107: rows of the broadcast mask, or None."""
    mask_shape, shape = tuple(mask_shape), tuple(shape)
    if len(mask_shape) > len(shape):
        return None
    padded = (1,) * (len(shape) - len(mask_shape)) + mask_shape
    if any(a != 1 and a != b for a, b in zip(padded, shape)):
        return None
    if all(n == 1 for n in padded):
        return 0
    if padded[-1] != shape[-1]:
        return None
    first = next(i for i, n in enumerate(padded) if n != 1)
    if padded[first:] != shape[first:]:
        return None
    rows = 1
    for n in padded[:-1]:
        rows *= n
    return rows


def allowed(shape, mask=None, causal=False, offset=0):
    """Boolean [rows, width] of allowed entries."""
    width = shape[-1]
    rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
    ok = np.ones((rows, width), bool)
    if causal:
        queries = max(1, shape[-2]) if len(shape) > 1 else 1
        q = np.arange(rows) % queries
        ok &= np.arange(width)[None, :] <= (min(offset, width) + q)[:, None]
    if mask is not None:
        mrows = mask_rows(mask.shape, shape)
        flat = np.asarray(mask, bool).reshape(-1, width) if mrows else np.asarray(mask, bool).reshape(1, width)
        ok &= flat[np.arange(rows) % mrows] if mrows else flat[0][None, :]
    return ok


def forward(x, mask=None, causal=False, offset=0):
    """(y, status) with status per row: 0 ok, 1 empty, 2 invalid."""
    x = np.asarray(x, np.float32)
    shape = x.shape
    width = shape[-1]
    v = x.reshape(-1, width).copy()
    ok = allowed(shape, mask, causal, offset)
    v[~ok] = -np.inf
    with np.errstate(invalid="ignore"):
        m = np.max(v, axis=1) if width else np.full(v.shape[0], -np.inf, np.float32)
    nan_row = np.isnan(v).any(axis=1)
    m = np.where(nan_row, np.float32(np.nan), m).astype(np.float32)
    empty = m == -np.inf
    invalid = np.isnan(m) | (m == np.inf)
    with np.errstate(over="ignore", under="ignore", invalid="ignore"):
        e = np.exp((v - m[:, None]).astype(np.float32)).astype(np.float32)
        e[empty] = 0
        e[invalid] = np.nan
        s = e.sum(axis=1, dtype=np.float32)
        y = (e / s[:, None]).astype(np.float32)
    y[empty] = 0
    status = np.where(empty, 1, np.where(invalid, 2, 0))
    return y.reshape(shape), status


def backward(y, g, mask=None, causal=False, offset=0):
    y = np.asarray(y, np.float32)
    g = np.asarray(g, np.float32)
    shape = y.shape
    width = shape[-1]
    yv, gv = y.reshape(-1, width), g.reshape(-1, width)
    dot = (gv * yv).sum(axis=1, dtype=np.float32)
    out = (yv * (gv - dot[:, None])).astype(np.float32)
    out[~allowed(shape, mask, causal, offset)] = 0
    return out.reshape(shape)
