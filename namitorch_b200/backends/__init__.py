"""Backend seam: the fused-kernel switch and the per-device CUDA backend object.

Mirrors namitorch/backends/__init__.py:32-48 (``get_backend``) and
namitorch/backends/_settings.py:1-12 (``enable_fused_kernels``). This build has one backend,
CUDA on sm_100a; asking for a CPU backend raises instead of falling back to NumPy.
"""
from __future__ import annotations

import threading

_fused_kernels_enabled = True
_lock = threading.RLock()
_backends: dict = {}


def enable_fused_kernels(mode):
    """namitorch/backends/_settings.py:4-8."""
    global _fused_kernels_enabled
    if type(mode) is not bool:
        raise TypeError("Fused kernel mode must be a Python bool.")
    _fused_kernels_enabled = mode


def fused_kernels_enabled():
    return _fused_kernels_enabled


def get_backend(value=None):
    """The CUDA backend of a tensor or device (namitorch/backends/__init__.py:32-48)."""
    import torch

    from .cuda import CUDABackend
    if isinstance(value, torch.Tensor):
        device = value.device
    elif value is None:
        device = torch.device("cuda", torch.cuda.current_device())
    else:
        device = torch.device(value)
    if device.type != "cuda":
        raise RuntimeError(f"namitorch_b200 has no {device.type} backend: its kernels run on CUDA devices only.")
    if device.index is None:
        device = torch.device("cuda", torch.cuda.current_device())
    with _lock:
        if device not in _backends:
            _backends[device] = CUDABackend(device)
        return _backends[device]


def try_fused(operation, *arrays):
    """namitorch/backends/__init__.py:55-60: the fused elementwise operation, or None when
    disabled or not applicable (the caller then uses its own path)."""
    if not fused_kernels_enabled():
        return None
    kernels = getattr(get_backend(arrays[0]), "fused", None)
    return None if kernels is None else kernels.run(operation, arrays)


def try_fused_softmax(operation, *arrays, **parameters):
    """namitorch/backends/__init__.py:63-68: the fused row softmax, or None when disabled or
    not applicable (the caller then uses its own path)."""
    if not fused_kernels_enabled():
        return None
    kernels = getattr(get_backend(arrays[0]), "softmax", None)
    return None if kernels is None else kernels.run(operation, arrays, **parameters)


def try_fused_normalization(operation, *arrays, **parameters):
    """namitorch/backends/__init__.py:71-76: the fused normalization, or None."""
    if not fused_kernels_enabled():
        return None
    kernels = getattr(get_backend(arrays[0]), "normalization", None)
    return None if kernels is None else kernels.run(operation, arrays, **parameters)


__all__ = ["enable_fused_kernels", "fused_kernels_enabled", "get_backend", "try_fused", "try_fused_softmax",
           "try_fused_normalization"]
