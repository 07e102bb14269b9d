"""Optimizers and gradient clipping of the hot path (namitorch.optim API)."""
from .adam import Adam, AdamW
from .clip_grad import clip_grad_norm_, clip_grad_value_, defer_gradient_transforms, get_grad_norm
from .optimizer import Optimizer
from . import lr_scheduler
from .lr_scheduler import Schedule, WarmupCosine

__all__ = ["Optimizer", "Adam", "AdamW", "clip_grad_norm_", "clip_grad_value_", "get_grad_norm",
           "defer_gradient_transforms", "lr_scheduler", "Schedule", "WarmupCosine"]
