"""Gradient-norm and gradient-value clipping (namitorch/optim/clip_grad.py:12-124).

``clip_grad_norm_`` keeps the reference's signature, validation and return value (a
float64 0-d tensor holding the pre-clip total norm), computed on the device by one
reduction kernel. When the parameters are exactly those (with gradients) of a
namitorch_b200 Adam/AdamW, the multiply by ``max_norm / (norm + 1e-6)`` is deferred into
that optimizer's next update, which reads the gradients anyway; otherwise the gradients
are rewritten in place, as the reference does. ``norm.item()`` or
``error_if_nonfinite=True`` synchronise with the device; nothing else does.
"""
from __future__ import annotations

import math
import operator
from numbers import Real

import numpy as np
import torch

from .. import _native as N
from ..flat import grad_stats_for, launch_transform
from .adam import _owner_of

_LAZY = True


def defer_gradient_transforms(mode: bool) -> None:
    """Whether clip_grad_norm_ / GradScaler.unscale_ may fold their factors into the next fused
    update instead of rewriting gradient storage (default True)."""
    global _LAZY
    if type(mode) is not bool:
        raise TypeError("defer_gradient_transforms mode must be a Python bool.")
    _LAZY = mode


def deferring_gradient_transforms() -> bool:
    return _LAZY


def _nonnegative(value: object, name: str) -> float:
    """namitorch/optim/clip_grad.py:12-21."""
    if isinstance(value, (bool, np.bool_)) or not isinstance(value, Real):
        raise TypeError(f"{name} must be a finite nonnegative real scalar.")
    try:
        value = float(value)
    except OverflowError:
        raise ValueError(f"{name} must be finite.") from None
    if not math.isfinite(value) or value < 0:
        raise ValueError(f"{name} must be finite and nonnegative.")
    return value


def _norm_type(value: object) -> float:
    """namitorch/optim/clip_grad.py:24-33."""
    if isinstance(value, (bool, np.bool_)) or not isinstance(value, Real):
        raise TypeError("norm_type must be a positive real scalar or positive infinity.")
    try:
        value = float(value)
    except OverflowError:
        raise ValueError("norm_type is outside the supported range.") from None
    if math.isnan(value) or value <= 0:
        raise ValueError("norm_type must be positive or positive infinity.")
    return value


_LAST_CHECKED = None   # (parameters, their gradients, the validated result) of the last call


def _parameters_and_gradients(parameters) -> tuple[list[torch.Tensor], list[torch.Tensor]]:
    """namitorch/optim/clip_grad.py:36-60 (gradients de-duplicated by identity). A call with the
    same parameter objects carrying the same gradient objects as the previous call reuses its
    validated result."""
    global _LAST_CHECKED
    if isinstance(parameters, torch.Tensor):
        parameters = (parameters,)
    if isinstance(parameters, (list, tuple)) or hasattr(parameters, "__next__"):
        items = list(parameters) if not isinstance(parameters, (list, tuple)) else parameters
        if all(type(p) is torch.nn.Parameter or type(p) is torch.Tensor for p in items):
            grads = [p.grad for p in items]
            last = _LAST_CHECKED
            if (last is not None and len(last[0]) == len(items) and all(map(operator.is_, last[0], items))
                    and all(map(operator.is_, last[1], grads))):
                return last[2]
            result = _validate_parameters(items)
            _LAST_CHECKED = (list(items), grads, result)
            return result
        parameters = items
    return _validate_parameters(parameters)


def _validate_parameters(parameters) -> tuple[list[torch.Tensor], list[torch.Tensor]]:
    if isinstance(parameters, (dict, str, bytes, set, frozenset)):
        raise TypeError("parameters must be a Tensor or an ordered iterable of Tensors.")
    try:
        parameters = iter(parameters)
    except TypeError:
        raise TypeError("parameters must be a Tensor or an ordered iterable of Tensors.") from None
    params, gradients = [], []
    seen = set()
    for parameter in parameters:
        if not isinstance(parameter, torch.Tensor):
            raise TypeError("parameters must contain only NamiTorch Tensors.")
        gradient = parameter.grad
        if gradient is None or id(gradient) in seen:
            continue
        if not isinstance(gradient, torch.Tensor) or not gradient.dtype.is_floating_point:
            raise TypeError("Gradients must be floating NamiTorch Tensors.")
        if gradient.shape != parameter.shape:
            raise ValueError(f"Gradient shape {tuple(gradient.shape)} does not match parameter shape "
                             f"{tuple(parameter.shape)}.")
        if gradient.device != parameter.device:
            raise RuntimeError(f"Operands are on different devices: {parameter.device}, {gradient.device}; "
                               "use an explicit .to() transfer.")
        seen.add(id(gradient))
        params.append(parameter)
        gradients.append(gradient)
    devices = {g.device for g in gradients}
    if len(devices) > 1:
        raise RuntimeError(f"Operands are on different devices: {', '.join(map(str, devices))}; "
                           "use an explicit .to() transfer.")
    return params, gradients


def _require_cuda(gradients: list[torch.Tensor]) -> None:
    if gradients and gradients[0].device.type != "cuda":
        raise RuntimeError("namitorch_b200 computes gradient norms on CUDA devices only.")


def _sole_owner(params: list[torch.Tensor]):
    """The optimizer whose gradients are exactly these parameters' gradients, if any."""
    if not params:
        return None
    owner = _owner_of(params[0])
    if owner is None or any(_owner_of(p) is not owner for p in params):
        return None
    entries = owner._entries()
    if {id(p) for _, p, _ in entries} != {id(p) for p in params}:
        return None
    return owner


def _sharded_owner(params: list[torch.Tensor]):
    """The ZeRO-1 optimizer that owns exactly these parameters, if any. Its gradients only
    mean something after its reduce-scatter, so the norm and the clips go through it."""
    owner = _sole_owner(params)
    return owner if owner is not None and getattr(owner, "_sharded", False) else None


def _pending_owners(params: list[torch.Tensor]):
    owners = {}
    for p in params:
        o = _owner_of(p)
        if o is not None and o._amp is not None:
            owners[id(o)] = o
    return list(owners.values())


def get_grad_norm(parameters, norm_type: float = 2) -> torch.Tensor:
    """namitorch/optim/clip_grad.py:86-88."""
    order = _norm_type(norm_type)
    params, gradients = _parameters_and_gradients(parameters)
    sharded = _sharded_owner(params)
    if sharded is not None:
        return sharded._grad_norm(order)[N.STATS_FIELDS.index("norm")]
    _require_cuda(gradients)
    for owner in _pending_owners(params):
        owner._materialize_pending()
    stats = grad_stats_for(gradients, norm_type=order)
    return stats[N.STATS_FIELDS.index("norm")]


def clip_grad_norm_(parameters, max_norm: float, norm_type: float = 2, error_if_nonfinite: bool = False):
    """namitorch/optim/clip_grad.py:96-112."""
    maximum = _nonnegative(max_norm, "max_norm")
    order = _norm_type(norm_type)
    if type(error_if_nonfinite) is not bool:
        raise TypeError("error_if_nonfinite must be a Python bool.")
    params, gradients = _parameters_and_gradients(parameters)
    norm_index = N.STATS_FIELDS.index("norm")

    def check(stats):
        if error_if_nonfinite:
            value = float(stats[norm_index].item())
            if not math.isfinite(value):
                raise RuntimeError(f"Cannot clip gradients with nonfinite total norm {value}.")

    sole = _sole_owner(params)
    sharded = sole if sole is not None and getattr(sole, "_sharded", False) else None
    owner = sharded if sharded is not None else (sole if _LAZY else None)
    stats = owner._lazy_clip(maximum, order, check) if owner is not None else None
    if stats is not None and sharded is not None and not _LAZY:
        sharded._materialize_pending()   # eager: rewrite the reduced shard now
    if stats is None:
        _require_cuda(gradients)
        for o in _pending_owners(params):
            o._materialize_pending()
        stats = grad_stats_for(gradients, norm_type=order)
        check(stats)
        launch_transform(gradients, stats=stats, max_norm=maximum)
    return stats[norm_index]


def clip_grad_value_(parameters, clip_value: float) -> None:
    """namitorch/optim/clip_grad.py:115-121."""
    bound = _nonnegative(clip_value, "clip_value")
    params, gradients = _parameters_and_gradients(parameters)
    sharded = _sharded_owner(params)
    if sharded is not None:
        sharded._clip_value_(bound)
        return
    _require_cuda(gradients)
    for owner in _pending_owners(params):
        owner._materialize_pending()
    launch_transform(gradients, clip_value=bound)


__all__ = ["get_grad_norm", "clip_grad_norm_", "clip_grad_value_", "defer_gradient_transforms"]
