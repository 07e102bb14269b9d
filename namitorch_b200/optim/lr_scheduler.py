"""Learning-rate schedules whose step can be gated on the device.

A schedule here is one function, ``lr_at(step, base_lr) -> lr`` (float64), applied to every
parameter group's base learning rate. ``Schedule`` runs any such function against an
optimizer; ``WarmupCosine``, the schedule the reference's training runner builds
(namitorch/training/runner.py:213), is provided. Its formula is the reference's
(namitorch/optim/lr_scheduler.py:248-269), evaluated in the same float64 operations and order,
so every learning rate is bit-identical to the reference's. The reference's other schedulers
(StepLR, MultiStepLR, ExponentialLR, CosineAnnealingLR, LinearLR) are not rebuilt here: pass
their formula as ``lr_at`` (with ``name`` and ``config`` for the state_dict).

Two ways to step:

* ``step()``: the host path. The groups' ``"lr"`` is rewritten, and the optimizer reads it
  on its next step, as in the reference.
* ``step(flag)`` with the flag ``GradScaler.step`` returned: the training loop's
  ``if updated: scheduler.step()`` (namitorch/training/runner.py:250-254) without a host
  read of found_inf. The step counter lives on the device, where ``nt_schedule_step`` adds 1
  when found_inf is 0, and the fused update reads each group's ``_scalar(lr)``,
  ``_scalar(1 - lr * weight_decay)`` and ``lr != 0`` from a table indexed by that counter
  (``nt_adamw_mt`` ``lr_schedule``). The host fills the table ahead of the counter: it knows
  an upper bound, one more per gated step.

Once the counter is on the device, the host view (``last_step``, ``get_last_lr()``, the
groups' ``"lr"``, ``state_dict()``) reads it when asked, which synchronises.

``state_dict()`` keeps the reference's version-1 fields (version, scheduler, last_step,
base_lrs, config), so a checkpoint's scheduler entry moves between the two.
"""
from __future__ import annotations

import math
from numbers import Integral, Real
from typing import Callable

import numpy as np
import torch

from .. import _native as N
from ._common import _scalar
from .optimizer import Optimizer

LrAt = Callable[[int, float], float]


# ---- argument checks (the reference's messages, so callers' error handling carries over) ----
def _count(value, name: str, least: int = 0) -> int:
    if isinstance(value, Integral) and not isinstance(value, bool):
        if int(value) >= least:
            return int(value)
        raise ValueError(f"{name} must be at least {least}.")
    raise TypeError(f"{name} must be an integer.")


def _rate(value, name: str) -> float:
    if isinstance(value, bool) or not isinstance(value, Real):
        raise TypeError(f"{name} must be a finite nonnegative real scalar.")
    try:
        out = float(value)
    except OverflowError:
        raise ValueError(f"{name} must be finite.") from None
    if math.isfinite(out) and out >= 0:
        return out
    raise ValueError(f"{name} must be finite and nonnegative.")


# ---- the device counter and its table --------------------------------------------------------
class _DeviceCounter:
    """The schedule's step on the device, and the per-step coefficient table the fused
    update reads (rows: steps; columns: parameter groups)."""

    ENTRY = np.dtype([("lr", "<f4"), ("decay", "<f4"), ("update", "<i4"), ("reserved", "<i4")])

    def __init__(self, schedule: "Schedule", device: torch.device):
        self.device = device
        self.step = torch.tensor([schedule._host_step], dtype=torch.int32, device=device)
        self.upper = schedule._host_step   # the counter never exceeds this
        self.table = None
        self.rows = 0
        self.key = None

    @staticmethod
    def _key(schedule: "Schedule"):
        optimizer = schedule.optimizer
        decoupled = bool(getattr(optimizer, "_decoupled_weight_decay", True))
        decays = tuple(float(group.get("weight_decay", 0.0)) for group in optimizer.param_groups)
        return decays, tuple(schedule.base_lrs), schedule._config_key(), decoupled

    def build(self, schedule: "Schedule", rows: int) -> None:
        decays, bases, _, decoupled = key = self._key(schedule)
        table = np.zeros((rows, len(decays)), dtype=self.ENTRY)
        for s in range(rows):
            for g, (lr, wd) in enumerate(zip(schedule._lrs(s), decays)):
                decay = _scalar(1 - lr * wd, "decay factor") if decoupled else 1.0
                table[s, g] = (_scalar(lr), decay, int(lr != 0), 0)
        self.table = torch.from_numpy(table.view(np.uint8).reshape(-1).copy()).to(self.device)
        self.rows = rows
        self.key = key

    def args(self, schedule: "Schedule"):
        """(table pointer, rows, columns, counter pointer) covering every value the counter
        can hold when the next update runs."""
        need = self.upper + 1
        if self.table is None or self._key(schedule) != self.key or need > self.rows:
            self.build(schedule, max(need, 2 * self.rows, 64))
        return self.table.data_ptr(), self.rows, len(schedule.optimizer.param_groups), self.step.data_ptr()


# ---- schedules ---------------------------------------------------------------------------------
class Schedule:
    """Runs ``lr_at(step, base_lr)`` for every parameter group of ``optimizer``.

    ``base_lrs`` are the groups' ``"initial_lr"`` (set by an earlier schedule) or ``"lr"``.
    Construction applies step ``last_step``. ``name`` and ``config`` are what ``state_dict``
    records; a state loads only into a schedule of the same name."""

    def __init__(self, optimizer: Optimizer, lr_at: LrAt, *, last_step: int = 0, name: str = "Schedule",
                 config: dict | None = None):
        if not isinstance(optimizer, Optimizer):
            raise TypeError("Scheduler optimizer must be a NamiTorch Optimizer.")
        if not callable(lr_at):
            raise TypeError("lr_at must be a callable (step, base_lr) -> lr.")
        optimizer._registered_parameters()
        bases = []
        for group in optimizer.param_groups:
            if "lr" not in group:
                raise ValueError("Every optimizer parameter group must define lr.")
            _rate(group["lr"], "lr")
            bases.append(_rate(group.get("initial_lr", group["lr"]), "initial_lr"))
        self.optimizer = optimizer
        self.base_lrs = bases
        self.name = name
        self.config = dict(config or {})
        self._lr_at = lr_at
        self._groups = self._group_ids()
        self._host_step = _count(last_step, "last_step")
        self._device: _DeviceCounter | None = None
        self._write(self._host_step)

    # ---- evaluation ------------------------------------------------------------------------
    def _lrs(self, step: int) -> list[float]:
        try:
            values = [self._lr_at(step, base) for base in self.base_lrs]
        except OverflowError:
            raise ValueError("Scheduled learning rate exceeds the finite supported range.") from None
        return [_rate(v, "scheduled lr") for v in values]

    def _write(self, step: int) -> None:
        values = self._lrs(step)
        for group, base, lr in zip(self.optimizer.param_groups, self.base_lrs, values):
            group["initial_lr"] = base
            group["lr"] = lr
        self._last_lr = values

    def _config_key(self):
        return repr(sorted(self.config.items()))

    def _group_ids(self):
        return [tuple(id(p) for p in group["params"]) for group in self.optimizer.param_groups]

    def _check_groups(self) -> None:
        self.optimizer._registered_parameters()
        if self._group_ids() != self._groups:
            raise RuntimeError("Optimizer parameter groups changed after scheduler construction; create a new scheduler.")

    # ---- host view ---------------------------------------------------------------------------
    def _pull(self) -> None:
        """Brings the device counter (if any) into the host state and the groups' lr."""
        if self._device is None:
            return
        step = int(self._device.step.item())
        self._device.upper = step
        if step != self._host_step:
            self._host_step = step
            self._write(step)

    @property
    def last_step(self) -> int:
        self._pull()
        return self._host_step

    @last_step.setter
    def last_step(self, value) -> None:
        self._host_step = _count(value, "last_step")
        if self._device is not None:
            self._device.step.fill_(self._host_step)
            self._device.upper = self._host_step

    def get_lr(self) -> list[float]:
        self._check_groups()
        return self._lrs(self.last_step)

    def get_last_lr(self) -> list[float]:
        self._pull()
        return list(self._last_lr)

    # ---- stepping ----------------------------------------------------------------------------
    def step(self, gate=None) -> None:
        """One schedule step. ``gate``: the flag ``GradScaler.step`` returned, or a bool; the
        step then counts only when the optimizer step was applied. A flag that has not been
        read on the host is decided on the device."""
        from ..amp import DeviceFlag
        if isinstance(gate, DeviceFlag) and gate._value is None:
            self._device_step(gate)
        elif gate is None or bool(gate):
            if self._device is not None:      # once on the device, the device counter leads
                self._device_step(None)
            else:
                self._check_groups()
                self._host_step += 1
                self._write(self._host_step)

    def _ensure_device_counter(self) -> _DeviceCounter:
        """Moves the step counter to the device (once) and attaches the table to the optimizer."""
        if self._device is None:
            device = self.optimizer._registered_parameters()[0].device
            if device.type != "cuda":
                raise RuntimeError("A device-gated scheduler step needs the optimizer on a CUDA device.")
            self._device = _DeviceCounter(self, device)
            self.optimizer._lr_schedule = self
        return self._device

    def _device_step(self, gate) -> None:
        self._check_groups()
        if gate is not None and not gate._invert:
            raise TypeError("step(gate) expects the flag GradScaler.step returned.")
        counter = self._ensure_device_counter()
        with torch.cuda.device(counter.device):
            if gate is None:
                N.call("nt_schedule_step", counter.step.data_ptr(), None, 0, N.stream_handle())
            else:
                flags = (N.C.c_void_p * 1)(gate._tensor.data_ptr())
                N.call("nt_schedule_step", counter.step.data_ptr(), flags, 1, N.stream_handle())
        counter.upper += 1

    def _schedule_args(self):
        """The device table for the optimizer's next fused update (None on the host path)."""
        return None if self._device is None else self._device.args(self)

    # ---- state -------------------------------------------------------------------------------
    def state_dict(self) -> dict:
        self.get_lr()
        return {"version": 1, "scheduler": self.name, "last_step": int(self.last_step),
                "base_lrs": list(self.base_lrs), "config": dict(self.config)}

    def _configure(self, config: dict) -> dict:
        """Checks a loaded config; a subclass with arguments validates and applies them."""
        if config != self.config:
            raise ValueError(f"{self.name} configuration must contain {tuple(self.config)}.")
        return config

    def load_state_dict(self, state: dict) -> None:
        self._check_groups()
        if not isinstance(state, dict):
            raise TypeError("Scheduler state must be a dictionary.")
        if set(state) != {"version", "scheduler", "last_step", "base_lrs", "config"}:
            raise ValueError("Invalid scheduler state fields.")
        if type(state["version"]) is not int or state["version"] != 1:
            raise ValueError("Unsupported scheduler state version.")
        if state["scheduler"] != self.name:
            raise ValueError("Saved scheduler type does not match the current scheduler.")
        step = _count(state["last_step"], "last_step")
        bases = state["base_lrs"]
        if not isinstance(bases, list) or len(bases) != len(self.optimizer.param_groups):
            raise ValueError("Saved base_lrs must match the optimizer parameter group count.")
        bases = [_rate(v, "base_lr") for v in bases]
        if not isinstance(state["config"], dict):
            raise ValueError(f"{self.name} configuration must contain {tuple(self.config)}.")
        old = (self.base_lrs, self.config)
        self.base_lrs, self.config = bases, self._configure(dict(state["config"]))
        try:
            self._lrs(step)
        except Exception:
            self.base_lrs, self.config = old
            raise
        self.last_step = step
        self._write(step)


class WarmupCosine(Schedule):
    """Linear warm-up from 0 over ``warmup_steps``, then a half cosine from each base lr down to
    ``min_lr`` at ``total_steps``, flat after it: the reference's WarmupCosine
    (namitorch/optim/lr_scheduler.py:248-269), same arguments, messages and float64 results."""

    def __init__(self, optimizer: Optimizer, warmup_steps: int, total_steps: int, min_lr: float = 0.0,
                 last_step: int = 0):
        config = self._checked(warmup_steps, total_steps, min_lr)
        super().__init__(optimizer, self._lr_at, last_step=last_step, name="WarmupCosine", config=config)

    @staticmethod
    def _checked(warmup_steps, total_steps, min_lr) -> dict:
        warmup = _count(warmup_steps, "warmup_steps")
        total = _count(total_steps, "total_steps", 1)
        if warmup >= total:
            raise ValueError("warmup_steps must be smaller than total_steps.")
        return {"warmup_steps": warmup, "total_steps": total, "min_lr": _rate(min_lr, "min_lr")}

    def _configure(self, config: dict) -> dict:
        if set(config) != {"warmup_steps", "total_steps", "min_lr"}:
            raise ValueError("WarmupCosine configuration must contain ('warmup_steps', 'total_steps', 'min_lr').")
        return self._checked(config["warmup_steps"], config["total_steps"], config["min_lr"])

    def _lrs(self, step: int) -> list[float]:
        if any(self.config["min_lr"] > base for base in self.base_lrs):
            raise ValueError("Minimum learning rate cannot exceed a group's base learning rate.")
        return super()._lrs(step)

    def _lr_at(self, step: int, base: float) -> float:
        warmup, total, floor = self.config["warmup_steps"], self.config["total_steps"], self.config["min_lr"]
        if step < warmup:
            return base * (step / warmup)
        progress = (min(step, total) - warmup) / (total - warmup)
        return floor + (base - floor) * ((1 + math.cos(math.pi * progress)) / 2)


__all__ = ["Schedule", "WarmupCosine"]
