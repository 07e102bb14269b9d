"""Learning-rate schedules restated in plain Python — TEST INFRASTRUCTURE ONLY.

Each function returns the reference scheduler's ``_compute_lrs(step, base_lrs, config)``
(namitorch/optim/lr_scheduler.py) for one step, in the same float64 arithmetic and order:
StepLR (:162-164), MultiStepLR (:188-190), ExponentialLR (:205-207), CosineAnnealingLR
(:223-225), LinearLR (:242-245), WarmupCosine (:264-269), with ``_floor_lrs`` (:30-33).
``gated_lrs`` replays the training loop's ``if updated: scheduler.step()``
(namitorch/training/runner.py:250-254): the lr each optimizer step uses.
"""
from __future__ import annotations

import math
from bisect import bisect_right


def floor_lrs(base_lrs, minimum, fraction):
    if any(minimum > base for base in base_lrs):
        raise ValueError("Minimum learning rate cannot exceed a group's base learning rate.")
    return [minimum + (base - minimum) * fraction for base in base_lrs]


def step_lr(step, base_lrs, step_size, gamma):
    factor = gamma ** (step // step_size)
    return [base * factor for base in base_lrs]


def multistep_lr(step, base_lrs, milestones, gamma):
    factor = gamma ** bisect_right(sorted(milestones), step)
    return [base * factor for base in base_lrs]


def exponential_lr(step, base_lrs, gamma):
    factor = gamma ** step
    return [base * factor for base in base_lrs]


def cosine_annealing_lr(step, base_lrs, T_max, eta_min):
    progress = min(step, T_max) / T_max
    return floor_lrs(base_lrs, eta_min, (1 + math.cos(math.pi * progress)) / 2)


def linear_lr(step, base_lrs, start_factor, end_factor, total_iters):
    progress = min(step, total_iters) / total_iters
    factor = start_factor * (1 - progress) + end_factor * progress
    return [base * factor for base in base_lrs]


def warmup_cosine(step, base_lrs, warmup_steps, total_steps, min_lr):
    floor_lrs(base_lrs, min_lr, 1.0)
    if step < warmup_steps:
        return [base * (step / warmup_steps) for base in base_lrs]
    progress = (min(step, total_steps) - warmup_steps) / (total_steps - warmup_steps)
    return floor_lrs(base_lrs, min_lr, (1 + math.cos(math.pi * progress)) / 2)


SCHEDULES = {"StepLR": step_lr, "MultiStepLR": multistep_lr, "ExponentialLR": exponential_lr,
             "CosineAnnealingLR": cosine_annealing_lr, "LinearLR": linear_lr, "WarmupCosine": warmup_cosine}


def lrs(name: str, step: int, base_lrs, config: dict):
    return SCHEDULES[name](step, base_lrs, **config)


def gated_lrs(name: str, base_lrs, config: dict, stepped: list[bool], last_step: int = 0):
    """The per-group lr used by each optimizer step when the scheduler advances only after
    applied steps; also returns the scheduler's final step."""
    step = last_step
    used = []
    for applied in stepped:
        used.append(lrs(name, step, base_lrs, config))
        if applied:
            step += 1
    return used, step
