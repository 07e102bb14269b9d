"""Adam / AdamW update, restated from the reference NumPy path — TEST INFRASTRUCTURE ONLY.

Follows, operation by operation and in float32:
* ``Adam._update_parameter``  namitorch/optim/adam.py:28-42
* ``_gradient``               namitorch/optim/_common.py:57-64
* ``_apply_update``           namitorch/optim/_common.py:67-73
* ``_scalar``                 namitorch/optim/_common.py:39-47 (float64 -> float32 coefficient)
* AdamW fused coefficients    namitorch/optim/adam.py:82-86 (identical expressions)

NumPy evaluates ``np.float32 scalar * float32 array`` in float32 with one rounding per
operation, so every line below is one IEEE float32 operation of the reference.
"""
from __future__ import annotations

import math
from concurrent.futures import ThreadPoolExecutor

import numpy as np

f32 = np.float32


def scalar(value: float, name: str = "coefficient") -> np.float32:
    """``_scalar`` (namitorch/optim/_common.py:39-47) for a float32 parameter."""
    if not math.isfinite(value) or abs(value) > float(np.finfo(np.float32).max):
        raise ValueError(f"Optimizer {name} must be representable in float32.")
    with np.errstate(under="ignore"):
        result = np.float32(value)
    if name == "eps" and result == 0:
        raise ValueError("Optimizer eps must remain positive in float32.")
    return result


def bias_corrections(beta1: float, beta2: float, step: int) -> tuple[np.float32, np.float32]:
    """f32(1 - beta1**step), f32(1 - beta2**step) (namitorch/optim/adam.py:38-39, :85)."""
    return scalar(1 - beta1 ** step), scalar(1 - beta2 ** step)


def adam_update(param: np.ndarray, grad: np.ndarray, exp_avg: np.ndarray, exp_avg_sq: np.ndarray,
                step: int, *, lr: float, beta1: float, beta2: float, eps: float, weight_decay: float,
                maximize: bool = False, decoupled: bool = True) -> int:
    """One update of one parameter, in place. Returns the new step count.

    ``step`` is the state's step before the update (``state.get("step", 0)``)."""
    # _gradient (namitorch/optim/_common.py:57-64)
    g = np.array(grad, dtype=np.float32, copy=True)
    if maximize:
        np.negative(g, out=g)
    if weight_decay != 0 and not decoupled:
        g += scalar(weight_decay) * param
    # moments (namitorch/optim/adam.py:35-36)
    exp_avg[...] = scalar(beta1) * exp_avg + scalar(1 - beta1) * g
    exp_avg_sq[...] = scalar(beta2) * exp_avg_sq + scalar(1 - beta2) * g * g
    step = step + 1
    corr1, corr2 = bias_corrections(beta1, beta2, step)
    # namitorch/optim/adam.py:39-42
    first_corrected = exp_avg / corr1
    second_corrected = exp_avg_sq / corr2
    denominator = np.sqrt(second_corrected) + scalar(eps, "eps")
    update = first_corrected / denominator
    # _apply_update (namitorch/optim/_common.py:67-73)
    if lr != 0:
        values = param
        if decoupled and weight_decay != 0:
            values = values * scalar(1 - lr * weight_decay, "decay factor")
        param[...] = values - scalar(lr) * update
    return step


def adamw_update_threaded(param, grad, exp_avg, exp_avg_sq, step, *, threads: int = 1, chunk: int = 1 << 22,
                          **options) -> int:
    """``adam_update`` over flat arrays, split into chunks that run on a thread pool.

    The update is elementwise, so chunking changes no result; NumPy ufuncs release the
    GIL, so the chunks run on separate cores. Used for the timed CPU baseline."""
    n = param.size
    if threads <= 1 or n <= chunk:
        return adam_update(param, grad, exp_avg, exp_avg_sq, step, **options)
    bounds = [(i, min(n, i + chunk)) for i in range(0, n, chunk)]

    def work(b):
        s, e = b
        adam_update(param[s:e], grad[s:e], exp_avg[s:e], exp_avg_sq[s:e], step, **options)

    with ThreadPoolExecutor(max_workers=threads) as pool:
        list(pool.map(work, bounds))
    return step + 1


class OracleAdamW:
    """Per-parameter AdamW state machine mirroring ``_FirstOrderOptimizer.step``
    (namitorch/optim/_common.py:133-167) for a list of float32 NumPy parameters.

    ``groups`` is a list of ``(indices, options)`` pairs; options hold lr, betas, eps,
    weight_decay and maximize. Parameters whose gradient is ``None`` are skipped, as
    ``_parameters_with_grad`` (namitorch/optim/optimizer.py:181-195) skips them."""

    def __init__(self, params: list[np.ndarray], groups, decoupled: bool = True):
        self.params = params
        self.groups = groups
        self.decoupled = decoupled
        self.state: dict[int, dict] = {}

    def step(self, grads: list[np.ndarray | None]) -> None:
        for indices, options in self.groups:
            beta1, beta2 = options["betas"]
            for i in indices:
                if grads[i] is None:
                    continue
                st = self.state.setdefault(i, {})
                if "exp_avg" not in st:
                    st["exp_avg"] = np.zeros_like(self.params[i])
                    st["exp_avg_sq"] = np.zeros_like(self.params[i])
                st["step"] = adam_update(
                    self.params[i], grads[i], st["exp_avg"], st["exp_avg_sq"], st.get("step", 0),
                    lr=options["lr"], beta1=beta1, beta2=beta2, eps=options["eps"],
                    weight_decay=options["weight_decay"], maximize=options.get("maximize", False),
                    decoupled=self.decoupled)
