"""``namitorch_b200.nn.functional`` holds the fused cross-entropy of the hot path."""
from . import functional

__all__ = ["functional"]
