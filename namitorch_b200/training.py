"""The training loop's optimizer tail, captured once as a CUDA graph and replayed.

The reference runs, every iteration (namitorch/training/runner.py:247-254),

    scaler.unscale_(optimizer)
    clip_grad_norm_(parameters, max_norm)
    updated = scaler.step(optimizer)
    scaler.update()
    if updated: scheduler.step()

With this package the tail already keeps every decision on the device: the loss scale and
growth tracker, found_inf and the skip, the clip coefficient, the per-parameter step counters
and bias corrections, and (with ``scheduler.step(updated)``) the learning-rate counter and
its schedule table. Its device work therefore does not depend on host values from one
iteration to the next, and ``CapturedOptimizerStep`` records it once as a CUDA graph. Each
call replays it: the host issues one graph launch instead of the tail's Python and kernel
launches, which is what bounds the small parameter sets (a 4M-parameter step is
microseconds of HBM traffic and a millisecond of host work).

What must hold across replays, and what the class sets up before capturing:

* the gradients are written in place into the same tensors every iteration (the flat
  gradient buffer's views, ``zero_grad(set_to_none=False)``), so their addresses are the ones
  recorded;
* the optimizer has taken one eager step (its moments and tables exist);
* the tables indexed by device counters are sized for ``capacity`` further steps at fixed
  addresses: the bias-correction table (it stops growing once the corrections round to 1)
  and the scheduler's learning-rate table.

Host mirrors that the eager path advances per call (the optimizer's step bound, the
scheduler's counter bound) are advanced per replay. The scaler is used as in the eager loop:
``scaler.scale(loss)`` before backward, then the replay instead of the tail.
"""
from __future__ import annotations

import contextlib
import threading

import torch

from .amp import GradScaler
from .optim.clip_grad import clip_grad_norm_

_capture = threading.local()


def capture_in_progress() -> bool:
    """True while CapturedOptimizerStep records the tail (the optimizer's step allows capture then)."""
    return bool(getattr(_capture, "active", False))


@contextlib.contextmanager
def _capturing():
    _capture.active = True
    try:
        yield
    finally:
        _capture.active = False


class CapturedOptimizerStep:
    """``unscale_ → clip_grad_norm_ → step → update → scheduler.step(updated)`` as one CUDA graph.

    ``optimizer``: a namitorch_b200 AdamW on the fused multi-tensor path, after one eager step.
    ``scaler``: a GradScaler (or None for a plain ``optimizer.step()``). ``parameters``: what
    ``clip_grad_norm_`` clips (default: the optimizer's parameters); ``max_norm`` None skips
    clipping. ``scheduler``: a scheduler stepped with the scaler's flag (or None).
    ``capacity``: replays the device tables are sized for; a replay past it raises.
    """

    def __init__(self, optimizer, scaler: GradScaler | None = None, parameters=None, *, max_norm=None,
                 norm_type: float = 2.0, scheduler=None, capacity: int = 10_000):
        if type(capacity) is not int or capacity < 1:
            raise ValueError("capacity must be a positive Python integer.")
        engine = getattr(optimizer, "_engine", None)
        uses_engine = getattr(optimizer, "_uses_engine", None)
        if engine is None or not callable(uses_engine) or not uses_engine():
            raise RuntimeError("CapturedOptimizerStep needs a namitorch_b200 optimizer on the fused multi-tensor "
                               "path that has taken one eager step.")
        if engine.exp_avg is None:
            raise RuntimeError("Take one eager optimizer step before capturing (the moments do not exist yet).")
        if scheduler is not None and scheduler.optimizer is not optimizer:
            raise ValueError("The scheduler must belong to the captured optimizer.")
        self.optimizer = optimizer
        self.scaler = scaler
        self.parameters = list(optimizer._registered_parameters()) if parameters is None else list(parameters)
        self.max_norm = max_norm
        self.norm_type = norm_type
        self.scheduler = scheduler
        self.capacity = capacity
        self.replays = 0
        self.norm = None
        self.updated = None
        device = engine.device
        with torch.cuda.device(device):
            # Tables the replays index by device counters, at their final size and address.
            engine.corrections.ensure(engine.max_step + capacity + 1)
            if scheduler is not None:
                counter = scheduler._ensure_device_counter()
                counter.build(scheduler, max(counter.rows, counter.upper + capacity + 2))
            torch.cuda.synchronize(device)
            if scaler is not None and scaler.is_enabled():
                scaler._scale_used = True   # the caller scales the loss before each replay
            step_bound = engine.max_step
            counter_bound = None if scheduler is None else scheduler._device.upper
            self.graph = torch.cuda.CUDAGraph()
            with _capturing(), torch.cuda.graph(self.graph):
                self._tail()
            # Capture recorded the device work without running it: undo the host mirrors' advance.
            engine.max_step = step_bound
            if scheduler is not None:
                scheduler._device.upper = counter_bound
            if scaler is not None:
                scaler._scale_used = False

    def _tail(self) -> None:
        scaler, optimizer = self.scaler, self.optimizer
        if scaler is not None:
            scaler.unscale_(optimizer)
        if self.max_norm is not None:
            self.norm = clip_grad_norm_(self.parameters, self.max_norm, self.norm_type)
        if scaler is not None:
            self.updated = scaler.step(optimizer)
            scaler.update()
        else:
            optimizer.step()
        if self.scheduler is not None:
            self.scheduler.step(self.updated)

    def __call__(self) -> None:
        """Replays the tail on the current stream's device (one graph launch)."""
        if self.replays >= self.capacity:
            raise RuntimeError(f"CapturedOptimizerStep was sized for {self.capacity} replays; capture a new one.")
        self.graph.replay()
        self.replays += 1
        self.optimizer._engine.max_step += 1
        if self.scheduler is not None:
            self.scheduler._device.upper += 1
        if self.scaler is not None:
            self.scaler._scale_used = False


__all__ = ["CapturedOptimizerStep", "capture_in_progress"]
