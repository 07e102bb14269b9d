"""RMS / layer normalization restated in NumPy float32 — TEST INFRASTRUCTURE ONLY.

Follows the reference's fused normalization kernels (namitorch/backends/cuda/
normalization.py:58-157): layer norm shifts each row by its first element, takes the mean
and the biased variance of the shifted values and saves (shifted mean, 1/sqrt(var + eps));
RMS norm saves (0, 1/sqrt(mean(x^2) + eps)); y = normalized * weight + bias. The backward
is the reference's normalization_backward (namitorch/autograd.py:575-601). Sums are NumPy's
float32 sums (pairwise), so results agree with any other summation order to float32
rounding, not bit for bit.
"""
from __future__ import annotations

import numpy as np


def forward(x, weight=None, bias=None, eps=1e-5, layer=True):
    x = np.asarray(x, np.float32)
    width = x.shape[-1]
    v = x.reshape(-1, width)
    e = np.float32(eps)
    if layer:
        d = (v - v[:, :1]).astype(np.float32)
        mean = (d.sum(axis=1, dtype=np.float32) / np.float32(width)).astype(np.float32)
        c = (d - mean[:, None]).astype(np.float32)
        var = ((c * c).sum(axis=1, dtype=np.float32) / np.float32(width)).astype(np.float32)
    else:
        c = v
        mean = np.zeros(v.shape[0], np.float32)
        var = ((v * v).sum(axis=1, dtype=np.float32) / np.float32(width)).astype(np.float32)
    inv = (np.float32(1) / np.sqrt((var + e).astype(np.float32))).astype(np.float32)
    y = (c * inv[:, None]).astype(np.float32)
    if weight is not None:
        y = (y * np.asarray(weight, np.float32)).astype(np.float32)
    if bias is not None:
        y = (y + np.asarray(bias, np.float32)).astype(np.float32)
    return y.reshape(x.shape), np.stack([mean, inv], axis=1).astype(np.float32)


def backward(x, weight, g, stats, layer=True):
    """(grad_input, grad_weight, grad_bias) from the saved statistics."""
    x = np.asarray(x, np.float32)
    width = x.shape[-1]
    v = x.reshape(-1, width)
    gv = np.asarray(g, np.float32).reshape(-1, width)
    mean, inv = stats[:, 0:1], stats[:, 1:2]
    centered = ((v - v[:, :1]) - mean) if layer else v
    n = (centered * inv).astype(np.float32)
    wg = gv if weight is None else (gv * np.asarray(weight, np.float32)).astype(np.float32)
    mp = (wg * n).mean(axis=1, keepdims=True, dtype=np.float32)
    local = wg - n * mp
    if layer:
        local = local - wg.mean(axis=1, keepdims=True, dtype=np.float32)
    dx = (inv * local).astype(np.float32)
    dw = (gv * n).sum(axis=0, dtype=np.float32)
    db = gv.sum(axis=0, dtype=np.float32)
    return dx.reshape(x.shape), dw, db
