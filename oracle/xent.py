"""Cross-entropy forward and backward, restated — TEST INFRASTRUCTURE ONLY.

Forward follows ``cross_entropy`` / ``_classification_loss`` / ``_class_loss_arguments``
(namitorch/nn/functional.py:792-863) with ``log_softmax`` computed as
``normalized_exponential_forward`` does (namitorch/_backend.py:321-354). The backward
applies the chain the reference autograd builds: mean / sum reduction, label smoothing
(confidence * loss + epsilon * smooth), class weights, the gather backward and the
log_softmax backward ``g - exp(out) * sum(g)`` with all-(-inf) rows zeroed
(namitorch/autograd.py:538-564). Everything is float32, as under ``float32_function``
(namitorch/amp.py:64-75).
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


def log_softmax(x: np.ndarray) -> np.ndarray:
    """``normalized_exponential_forward('log_softmax', x, (-1,))`` (namitorch/_backend.py:331-348)."""
    maximum = np.max(x, axis=-1, keepdims=True, initial=-np.inf)
    shifted = np.full_like(x, np.nan)
    with np.errstate(over="ignore", invalid="ignore"):
        np.subtract(x, maximum, out=shifted, where=np.isfinite(maximum))
    np.copyto(shifted, -np.inf, where=np.isneginf(maximum))
    with np.errstate(under="ignore"):
        exponentials = np.exp(shifted)
    denominator = np.sum(exponentials, axis=-1, keepdims=True, dtype=x.dtype)
    log_denominator = np.zeros_like(denominator)
    with np.errstate(divide="ignore"):
        np.log(denominator, out=log_denominator, where=denominator != 0)
    with np.errstate(over="ignore", invalid="ignore"):
        return np.asarray(shifted - log_denominator)


def cross_entropy(logits: np.ndarray, targets: np.ndarray, weight: np.ndarray | None = None,
                  ignore_index: int = -100, reduction: str = "mean", label_smoothing: float = 0.0,
                  with_grad: bool = True):
    """Returns (loss, dlogits) for a unit upstream gradient (ones per row for 'none').

    ``logits`` is float32 [N, C]; ``targets`` int64 [N]. ``loss`` is a float32 scalar, or
    a float32 [N] vector for reduction 'none'."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    n, classes = x.shape
    t = np.asarray(targets, dtype=np.int64).reshape(-1)
    valid = t != ignore_index
    selected = t[valid]
    if np.any(selected < 0) or np.any(selected >= classes):
        raise IndexError(f"Every non-ignored target must be in [0, {classes}).")
    positions = np.flatnonzero(valid)
    w = None if weight is None else np.asarray(weight, dtype=np.float32)
    example_w = None if w is None else w[selected]
    denominator = f32(selected.size) if w is None else np.sum(example_w, dtype=np.float32)
    grad = np.zeros_like(x) if with_grad else None
    if reduction == "mean" and denominator == 0:
        return (f32(0.0), grad)
    sel = x[positions]
    lp = log_softmax(sel)
    rows = np.arange(selected.size)
    with np.errstate(over="ignore", invalid="ignore"):
        loss_vec = -lp[rows, selected]
        if example_w is not None:
            loss_vec = loss_vec * example_w
        eps = f32(label_smoothing)
        if label_smoothing != 0:
            weighted = lp if w is None else lp * w
            smooth = -np.mean(weighted, axis=-1, dtype=np.float32)
            loss_vec = f32(1 - label_smoothing) * loss_vec + eps * smooth
    if reduction == "none":
        loss = np.zeros(n, dtype=np.float32)
        np.add.at(loss, positions, loss_vec)
    elif reduction == "sum":
        loss = np.sum(loss_vec, dtype=np.float32)
    else:
        loss = f32(np.sum(loss_vec, dtype=np.float32) / denominator)
    if not with_grad:
        return loss, None

    # Backward, upstream gradient 1 (per row for 'none').
    with np.errstate(over="ignore", invalid="ignore", under="ignore"):
        if reduction == "mean":
            g_rows = np.full(selected.size, f32(1.0) / denominator, dtype=np.float32)
        else:
            g_rows = np.ones(selected.size, dtype=np.float32)
        g_nll = g_rows * f32(1 - label_smoothing) if label_smoothing != 0 else g_rows
        dlp = np.zeros_like(lp)
        contrib = -g_nll if example_w is None else -(g_nll * example_w)
        dlp[rows, selected] += contrib
        if label_smoothing != 0:
            g_smooth = -(g_rows * eps) / f32(classes)
            if w is None:
                dlp += g_smooth[:, None]
            else:
                dlp += g_smooth[:, None] * w[None, :]
        total = np.sum(dlp, axis=-1, keepdims=True, dtype=np.float32)
        dx = dlp - np.exp(lp) * total
        dx[np.all(np.isneginf(lp), axis=-1)] = 0
    grad[positions] = dx
    return loss, grad
