"""CUDA backend object and the per-tensor AdamW kernel seam.

``AdamWCUDAKernel`` keeps the interface of the reference's ``backend.adamw``
(namitorch/backends/cuda/adamw.py:32-73): ``supports(...)`` answers whether four arrays can
take the fused update, ``run(...)`` validates the ten float32 coefficients and launches one
update on the current stream, returning False for an empty parameter. The arrays are torch
CUDA tensors; the kernel is ``nt_adamw_f32`` of libnamitorch_b200.so.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from .. import _native as N


class AdamWCUDAKernel:
    def __init__(self, backend=None):
        self._backend = backend

    @staticmethod
    def supports(parameter, gradient, first=None, second=None) -> bool:
        """namitorch/backends/cuda/adamw.py:33-46."""
        if parameter is None or gradient is None:
            return False
        present = [a for a in (parameter, gradient, first, second) if a is not None]
        for array in present:
            if not isinstance(array, torch.Tensor) or array.device.type != "cuda":
                return False
            if array.device != parameter.device or array.dtype != torch.float32:
                return False
            if not array.is_contiguous() or array.data_ptr() % 4 or array.shape != parameter.shape:
                return False
        ranges = [(a.data_ptr(), a.data_ptr() + a.numel() * 4) for a in present if a.numel()]
        return not any(max(s, os_) < min(e, oe) for i, (s, e) in enumerate(ranges) for os_, oe in ranges[i + 1:])

    def run(self, parameter, gradient, first, second, *, coefficients, maximize, update_parameter) -> bool:
        """namitorch/backends/cuda/adamw.py:54-73."""
        if first is None or second is None or not self.supports(parameter, gradient, first, second):
            raise RuntimeError("Fused AdamW requires non-overlapping contiguous float32 CUDA arrays with identical "
                               "shapes and device.")
        if len(coefficients) != 10 or any(not isinstance(v, np.float32) or not np.isfinite(v) for v in coefficients):
            raise ValueError("Fused AdamW requires ten finite float32 coefficients.")
        if coefficients[5] <= 0 or coefficients[8] <= 0 or coefficients[9] <= 0:
            raise ValueError("Fused AdamW eps and bias corrections must be positive.")
        if type(maximize) is not bool or type(update_parameter) is not bool:
            raise TypeError("Fused AdamW flags must be Python bools.")
        if parameter.numel() == 0:
            return False
        coef = (C.c_float * 10)(*[float(v) for v in coefficients])
        with torch.cuda.device(parameter.device):
            N.call("nt_adamw_f32", parameter.data_ptr(), gradient.data_ptr(), first.data_ptr(), second.data_ptr(),
                   coef, int(maximize), int(update_parameter), parameter.numel(), N.stream_handle())
        return True


class CUDABackend:
    """One per device (namitorch/backends/cuda/__init__.py:23-45); ``adamw``, ``fused``,
    ``softmax`` and ``normalization`` are the plugin seams."""

    def __init__(self, device: torch.device):
        N.load()
        self.device = device
        self.adamw = AdamWCUDAKernel(self)
        from .fused import FusedCUDAKernels
        from .normalization import NormalizationCUDAKernels
        from .softmax import SoftmaxCUDAKernels
        self.fused = FusedCUDAKernels(self)
        self.softmax = SoftmaxCUDAKernels(self)
        self.normalization = NormalizationCUDAKernels(self)

    @staticmethod
    def supports_float16() -> bool:
        return True

    @staticmethod
    def supports_bfloat16() -> bool:
        return True

    def __repr__(self) -> str:
        return f"CUDABackend({self.device})"
