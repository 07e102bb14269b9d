"""Mixed precision: autocast policy and a device-resident GradScaler.

API of namitorch/amp.py:18-262. Differences that follow from keeping the loss scale on the
GPU (so that no step of the AMP loop waits for the host):

* the scale and growth tracker are device tensors; ``update()`` is one tiny kernel
  (``nt_scaler_update``) implementing namitorch/amp.py:219-234 bit for bit;
* ``unscale_`` computes found_inf and the gradient norm with one reduction kernel. With
  deferred transforms (the default, see ``optim.defer_gradient_transforms``) it leaves the
  gradient storage untouched and the optimizer's fused update divides by the scale as it
  reads each gradient; otherwise it rewrites the gradients like the reference;
* ``unscale_`` and ``step`` return a ``DeviceFlag`` — truthy exactly when the reference
  would return True — which reads the device only when converted to bool;
* ``get_scale()`` and ``state_dict()`` synchronise (they return host values).

``autocast`` accepts float16 (the reference's only choice) and bfloat16.
"""
from __future__ import annotations

import math
import operator
from contextlib import contextmanager
from contextvars import ContextVar
from functools import wraps
from numbers import Real
from types import MappingProxyType

import numpy as np
import torch

from . import _native as N

OPERATION_POLICIES = MappingProxyType({
    "matmul": "low",
    "linear": "low",
    **dict.fromkeys(("sum", "mean", "prod", "var", "std", "logsumexp", "softmax", "log_softmax", "layer_norm",
                     "rms_norm", "batch_norm", "cross_entropy", "nll_loss", "mse_loss", "l1_loss", "smooth_l1_loss",
                     "huber_loss", "binary_cross_entropy", "binary_cross_entropy_with_logits", "exp", "expm1", "log",
                     "log1p", "log2", "log10", "sqrt", "rsqrt", "gelu", "sigmoid", "silu", "softplus", "softsign"),
                    "float32"),
})
_autocast_state = ContextVar("namitorch_b200_autocast", default=(False, torch.float16))
_LOW = (torch.float16, torch.bfloat16)


def _normalize_dtype(dtype) -> torch.dtype:
    if dtype in _LOW:
        return dtype
    names = {"float16": torch.float16, "half": torch.float16, "bfloat16": torch.bfloat16}
    if isinstance(dtype, str) and dtype in names:
        return names[dtype]
    raise ValueError("autocast supports float16 and bfloat16 compute dtypes.")


@contextmanager
def autocast(device_type="cuda", dtype=torch.float16, enabled=True):
    """namitorch/amp.py:26-48 (plus bfloat16)."""
    if device_type not in ("cpu", "cuda"):
        raise ValueError("autocast device_type must be 'cuda' or 'cpu'.")
    if type(enabled) is not bool:
        raise TypeError("autocast enabled must be a Python bool.")
    selected = _normalize_dtype(dtype)
    if device_type == "cpu":
        if enabled:
            raise RuntimeError("CPU autocast is not supported; use explicit Tensor.to(dtype) conversions.")
        yield
        return
    token = _autocast_state.set((enabled, selected))
    try:
        yield
    finally:
        _autocast_state.reset(token)


def autocast_dtype(operation, *operands):
    """The low-precision dtype an operation runs in under autocast, or None (namitorch/amp.py:51-61)."""
    enabled, dtype = _autocast_state.get()
    values = tuple(v for v in operands if v is not None)
    if not enabled or OPERATION_POLICIES.get(operation) != "low" or not values:
        return None
    if any(v.device.type != "cuda" or v.dtype not in (torch.float16, torch.bfloat16, torch.float32) for v in values):
        return None
    return dtype


def autocast_operands(operation, *operands):
    """The operands an operation computes with under autocast (namitorch/nn/functional.py:57-60):
    each non-None operand converted to ``autocast_dtype(operation, ...)`` when that is not None,
    else returned as given. A conversion to the dtype a tensor already has returns the tensor
    itself, so the parameters of an optimizer built with ``model_dtype`` (views of its
    persistent low-precision copy) pass through without the per-forward weight cast the
    reference makes."""
    dtype = autocast_dtype(operation, *operands)
    if dtype is None:
        return operands
    return tuple(None if value is None else value.to(dtype) for value in operands)


def float32_function(function):
    """Promotes float16 / bfloat16 tensor arguments to float32 (namitorch/amp.py:64-75)."""
    if OPERATION_POLICIES.get(function.__name__) != "float32":
        raise ValueError(f"No float32 policy for {function.__name__}.")

    def promote(value):
        return value.to(torch.float32) if isinstance(value, torch.Tensor) and value.dtype in _LOW else value

    @wraps(function)
    def checked(*args, **kwargs):
        return function(*(promote(v) for v in args), **{k: promote(v) for k, v in kwargs.items()})

    return checked


class DeviceFlag:
    """A boolean that lives on the device; ``bool(flag)`` synchronises and reads it."""

    __slots__ = ("_tensor", "_invert", "_value")

    def __init__(self, tensor: torch.Tensor | None, invert: bool = False, value: bool | None = None):
        self._tensor = tensor
        self._invert = invert
        self._value = value

    def __bool__(self) -> bool:
        if self._value is None:
            raw = bool(self._tensor.item() != 0)
            self._value = (not raw) if self._invert else raw
        return self._value

    def __eq__(self, other):
        return bool(self) == bool(other)

    def __hash__(self):
        return hash(bool(self))

    def __repr__(self) -> str:
        return f"DeviceFlag({bool(self)})"


class GradScaler:
    _MIN_SCALE = float(np.finfo(np.float32).tiny)
    _MAX_SCALE = float(np.finfo(np.float32).max)

    def __init__(self, init_scale=65536.0, growth_factor=2.0, backoff_factor=0.5, growth_interval=2000, enabled=True):
        """namitorch/amp.py:82-100."""
        if type(enabled) is not bool:
            raise TypeError("GradScaler enabled must be a Python bool.")
        self._init_value = self._scale_value(init_scale)
        self._growth_factor = self._real(growth_factor, "growth_factor")
        self._backoff_factor = self._real(backoff_factor, "backoff_factor")
        if self._growth_factor <= 1:
            raise ValueError("growth_factor must be greater than 1.")
        if not 0 < self._backoff_factor < 1:
            raise ValueError("backoff_factor must be between 0 and 1.")
        if isinstance(growth_interval, (bool, np.bool_)):
            raise TypeError("growth_interval must be a positive integer.")
        self._growth_interval = operator.index(growth_interval)
        if self._growth_interval <= 0:
            raise ValueError("growth_interval must be positive.")
        self._enabled = enabled
        self._init_tracker = 0
        self._scale_dev: torch.Tensor | None = None
        self._tracker_dev: torch.Tensor | None = None
        self._optimizer_states: dict[int, dict] = {}
        self._scale_used = False

    @staticmethod
    def _real(value, name):
        if isinstance(value, (bool, np.bool_)) or not isinstance(value, Real):
            raise TypeError(f"{name} must be a finite real number.")
        try:
            result = float(value)
        except OverflowError:
            raise ValueError(f"{name} must be finite.") from None
        if not math.isfinite(result):
            raise ValueError(f"{name} must be finite.")
        return result

    @classmethod
    def _scale_value(cls, value):
        """namitorch/amp.py:115-119."""
        scale = cls._real(value, "scale")
        if not cls._MIN_SCALE <= scale <= cls._MAX_SCALE:
            raise ValueError(f"scale must be between {cls._MIN_SCALE} and {cls._MAX_SCALE}.")
        return float(np.float32(scale))

    def _device_state(self, device: torch.device) -> torch.Tensor:
        if self._scale_dev is None:
            self._scale_dev = torch.tensor([self._init_value], dtype=torch.float32, device=device)
            self._tracker_dev = torch.tensor([self._init_tracker], dtype=torch.int32, device=device)
        elif self._scale_dev.device != device:
            raise RuntimeError(f"GradScaler state lives on {self._scale_dev.device}; got tensors on {device}.")
        return self._scale_dev

    @property
    def scale_tensor(self) -> torch.Tensor | None:
        """The device float32 [1] loss scale (None before first use)."""
        return self._scale_dev

    def is_enabled(self):
        return self._enabled

    def get_scale(self):
        if not self._enabled:
            return 1.0
        if self._scale_dev is None:
            return self._init_value
        return float(self._scale_dev.item())

    def scale(self, loss):
        """namitorch/amp.py:127-140: loss * scale, on the device."""
        if not isinstance(loss, torch.Tensor) or not loss.dtype.is_floating_point:
            raise TypeError("GradScaler.scale requires a floating NamiTorch Tensor.")
        if not self._enabled:
            return loss
        if self._optimizer_states:
            raise RuntimeError("Call update() before scaling another loss after unscale_ or step.")
        if loss.device.type != "cuda":
            raise RuntimeError("namitorch_b200 GradScaler keeps its scale on a CUDA device; the loss is on "
                               f"{loss.device}.")
        scale = self._device_state(loss.device)
        self._scale_used = True
        return loss * scale[0].to(loss.dtype)

    @staticmethod
    def _gradients(optimizer):
        if not callable(getattr(optimizer, "_parameters_with_grad", None)) or not callable(getattr(optimizer, "step", None)):
            raise TypeError("GradScaler requires a NamiTorch optimizer.")
        if not callable(getattr(optimizer, "_amp_unscale_", None)):
            raise TypeError("GradScaler requires a namitorch_b200 optimizer.")
        entries_of = getattr(optimizer, "_grad_entries", None)
        if entries_of is None:   # any optimizer exposing the reference's gradient walk
            entries = [(None, group, p, g) for group, p, g in optimizer._parameters_with_grad()]
        else:
            entries = entries_of()
            cached = getattr(optimizer, "_scaler_gradients", None)
            if cached is not None and cached[0] is entries:
                return cached[1]
        gradients = tuple((p, g) for _, _, p, g in entries)
        for p, g in gradients:
            if not p.dtype.is_floating_point or g.requires_grad or g.grad_fn is not None:
                raise RuntimeError("GradScaler requires detached floating gradients.")
        if entries_of is not None:
            optimizer._scaler_gradients = (entries, gradients)   # valid while the entries list is
        return gradients

    def unscale_(self, optimizer):
        """namitorch/amp.py:169-194."""
        if not self._enabled:
            return True
        if not self._scale_used:
            raise RuntimeError("Call scale(loss) and backward before unscale_.")
        identity = id(optimizer)
        if identity in self._optimizer_states:
            raise RuntimeError("unscale_ may be called only once per optimizer between update() calls.")
        gradients = self._gradients(optimizer)
        if not gradients:
            raise RuntimeError("No gradients were found for this optimizer.")
        previous = {id(p) for state in self._optimizer_states.values() for p, _ in state["gradients"]}
        if any(id(p) in previous for p, _ in gradients):
            raise RuntimeError("Optimizers cannot share gradients in the same GradScaler iteration.")
        from .optim.clip_grad import deferring_gradient_transforms
        state = {"optimizer": optimizer, "stage": "unscaling", "gradients": gradients, "stats": None}
        self._optimizer_states[identity] = state
        scale = self._device_state(gradients[0][1].device)
        stats = optimizer._amp_unscale_(scale, lazy=deferring_gradient_transforms())
        state["stats"] = stats
        state["stage"] = "unscaled"
        return DeviceFlag(stats[N.STATS_FIELDS.index("found_inf")], invert=True)

    def step(self, optimizer):
        """namitorch/amp.py:196-217; the skip decision stays on the device."""
        if not self._enabled:
            optimizer.step()
            return True
        identity = id(optimizer)
        if identity not in self._optimizer_states:
            self.unscale_(optimizer)
        state = self._optimizer_states[identity]
        if state["stage"] != "unscaled":
            raise RuntimeError("step() may be called only once per optimizer before update().")
        current = self._gradients(optimizer)
        if len(current) != len(state["gradients"]) or any(
                a[0] is not b[0] or a[1] is not b[1] for a, b in zip(current, state["gradients"])):
            raise RuntimeError("Optimizer gradients changed after unscale_; clipping must modify the existing "
                               "gradients in-place.")
        state["stage"] = "stepping"
        optimizer._amp_enable_skip()
        optimizer.step()
        state["stage"] = "stepped"
        return DeviceFlag(state["stats"][N.STATS_FIELDS.index("found_inf")], invert=True)

    def update(self):
        """namitorch/amp.py:219-234 as one device kernel."""
        if not self._enabled:
            return
        if not self._optimizer_states or any(s["stage"] != "stepped" for s in self._optimizer_states.values()):
            raise RuntimeError("Call step() for every unscaled optimizer before update().")
        found = [s["stats"][N.STATS_FIELDS.index("found_inf")].data_ptr() for s in self._optimizer_states.values()]
        if len(found) > N.NT_MAX_FOUND_INF:
            raise RuntimeError(f"GradScaler.update combines at most {N.NT_MAX_FOUND_INF} optimizers.")
        array = (N.C.c_void_p * len(found))(*found)
        with torch.cuda.device(self._scale_dev.device):
            N.call("nt_scaler_update", self._scale_dev.data_ptr(), self._tracker_dev.data_ptr(), array, len(found),
                   self._growth_factor, self._backoff_factor, self._growth_interval, N.stream_handle())
        self._optimizer_states.clear()
        self._scale_used = False

    def _ensure_idle(self):
        if self._optimizer_states or self._scale_used:
            raise RuntimeError("GradScaler state can be saved or loaded only between iterations, after update().")

    def state_dict(self):
        """namitorch/amp.py:240-242 (host values; synchronises)."""
        self._ensure_idle()
        scale = self._init_value if self._scale_dev is None else float(self._scale_dev.item())
        tracker = self._init_tracker if self._tracker_dev is None else int(self._tracker_dev.item())
        return dict(version=1, scale=scale, growth_factor=self._growth_factor, backoff_factor=self._backoff_factor,
                    growth_interval=self._growth_interval, enabled=self._enabled, growth_tracker=tracker)

    def load_state_dict(self, state):
        """namitorch/amp.py:244-262."""
        self._ensure_idle()
        if type(state) is not dict or set(state) != {"version", "scale", "growth_factor", "backoff_factor",
                                                     "growth_interval", "enabled", "growth_tracker"}:
            raise ValueError("Invalid GradScaler state fields.")
        if type(state["version"]) is not int or state["version"] != 1:
            raise ValueError("Unsupported GradScaler state version.")
        prepared = GradScaler(state["scale"], state["growth_factor"], state["backoff_factor"],
                              state["growth_interval"], state["enabled"])
        tracker = state["growth_tracker"]
        if type(tracker) is not int or not 0 <= tracker < prepared._growth_interval:
            raise ValueError("Invalid GradScaler growth_tracker.")
        self._init_value = prepared._init_value
        self._growth_factor = prepared._growth_factor
        self._backoff_factor = prepared._backoff_factor
        self._growth_interval = prepared._growth_interval
        self._enabled = prepared._enabled
        self._init_tracker = tracker
        if self._scale_dev is not None:
            self._scale_dev.fill_(self._init_value)
            self._tracker_dev.fill_(tracker)


__all__ = ["autocast", "autocast_dtype", "autocast_operands", "float32_function", "GradScaler", "DeviceFlag", "OPERATION_POLICIES"]
