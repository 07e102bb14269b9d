"""GradScaler arithmetic and the AMP optimizer step, restated — TEST INFRASTRUCTURE ONLY.

Follows ``GradScaler`` (namitorch/amp.py:78-262): ``_scale_value`` (:238-243),
``unscale_`` (:293-318: g = f32(g) / scale written back in the gradient dtype),
``_finite`` (:276-291), ``step`` (:320-341) and ``update`` (:343-358), plus the training
loop order of namitorch/training/runner.py:247-254 (unscale_, clip only when finite,
step, update).
"""
from __future__ import annotations

import math

import numpy as np

from . import clip as _clip
from .adamw import OracleAdamW

MIN_SCALE = float(np.finfo(np.float32).tiny)
MAX_SCALE = float(np.finfo(np.float32).max)


def scale_value(value: float) -> float:
    """``GradScaler._scale_value``: a float32-representable scale in [tiny, max]."""
    scale = float(value)
    if not math.isfinite(scale) or not MIN_SCALE <= scale <= MAX_SCALE:
        raise ValueError(f"scale must be between {MIN_SCALE} and {MAX_SCALE}.")
    return float(np.float32(scale))


class OracleGradScaler:
    def __init__(self, init_scale=65536.0, growth_factor=2.0, backoff_factor=0.5, growth_interval=2000):
        self.scale = scale_value(init_scale)
        self.growth_factor = float(growth_factor)
        self.backoff_factor = float(backoff_factor)
        self.growth_interval = int(growth_interval)
        self.growth_tracker = 0

    def unscale(self, grads: list[np.ndarray | None]) -> bool:
        """g = g / scale in float32, written back in place; returns all-finite."""
        finite = True
        with np.errstate(over="ignore", under="ignore", invalid="ignore"):
            for g in grads:
                if g is None:
                    continue
                g[...] = np.divide(g.astype(np.float32, copy=False), self.scale).astype(g.dtype)
        for g in grads:
            if g is not None:
                finite = finite and bool(np.all(np.isfinite(g)))
        return finite

    def update(self, found_inf: bool) -> None:
        if found_inf:
            self.scale = scale_value(max(MIN_SCALE, self.scale * self.backoff_factor))
            self.growth_tracker = 0
        else:
            self.growth_tracker += 1
            if self.growth_tracker == self.growth_interval:
                self.scale = scale_value(min(MAX_SCALE, self.scale * self.growth_factor))
                self.growth_tracker = 0


def amp_step(optimizer: OracleAdamW, scaler: OracleGradScaler, grads: list[np.ndarray | None],
             max_norm: float | None = None, norm_type: float = 2.0, storage=None, given_norm: float | None = None) -> dict:
    """One AMP iteration on float32 gradients that hold loss-scaled values.

    ``storage`` (float32 array -> float32 array) models gradients that live in a narrower
    dtype: ``unscale_`` and ``clip_grad_norm_`` write their results back into the gradient
    tensors in place (amp.py:186-191, clip_grad.py:106-111), so each result is rounded to
    that dtype before the next operation reads it (e.g. ``casts.round_to_bf16``).

    ``given_norm`` is passed to ``clip.clip_grad_norm_`` as the norm to clip with.

    Returns the scale that was used, whether the optimizer stepped, the pre-clip norm
    (None when clipping did not run) and the scale after ``update``."""
    def store():
        if storage is not None:
            for g in grads:
                if g is not None:
                    g[...] = storage(g)

    used = scaler.scale
    finite = scaler.unscale(grads)
    store()
    norm = None
    if finite and max_norm is not None:
        norm = float(_clip.clip_grad_norm_([g for g in grads if g is not None], max_norm, norm_type,
                                           error_if_nonfinite=True, norm=given_norm))
        store()
    if finite:
        optimizer.step(grads)
    scaler.update(not finite)
    return {"scale_used": used, "stepped": finite, "norm": norm, "scale_after": scaler.scale,
            "growth_tracker": scaler.growth_tracker}
