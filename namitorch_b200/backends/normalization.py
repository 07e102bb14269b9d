"""The normalization plugin seam (namitorch/backends/cuda/normalization.py:160-235) on torch tensors.

``NormalizationCUDAKernels.supports(operation, arrays)`` and ``run(operation, arrays, *,
eps=None, save_stats=True, needs=(True, True, True))`` keep the reference's operations
(``rms_norm``, ``layer_norm`` and their ``_backward``), argument checks and results: the
forward returns ``(output, statistics)`` with statistics ``[rows, 2]`` float32 (None unless
``save_stats``), the backward ``(grad_input, grad_weight, grad_bias)`` with None for the
gradients ``needs`` leaves out. ``run`` returns None when the arrays are not supported. The
kernels are ``nt_norm_forward`` / ``nt_norm_backward``. Besides float32 (the reference's only
dtype) they take float16 and bfloat16 tensors, computed in float32.
"""
from __future__ import annotations

import math

import numpy as np
import torch

from .. import _native as N

_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


class NormalizationCUDAKernels:
    def __init__(self, backend=None):
        self._backend = backend

    @staticmethod
    def _ok(array, like=None) -> bool:
        if not isinstance(array, torch.Tensor) or array.device.type != "cuda" or not array.is_contiguous():
            return False
        if like is not None and (array.device != like.device or array.dtype != like.dtype):
            return False
        return array.dtype in _DTYPES and array.data_ptr() % array.element_size() == 0

    def supports(self, operation, arrays) -> bool:
        """namitorch/backends/cuda/normalization.py:163-175."""
        backward = operation.endswith("_backward")
        name = operation.removesuffix("_backward")
        if name not in N.NORM_OPS or len(arrays) != (4 if backward else 3):
            return False
        value, weight = arrays[:2]
        if not self._ok(value) or value.dim() < 1 or not 1 <= value.shape[-1] <= N.NT_NORM_MAX_WIDTH:
            return False
        if weight is not None and (not self._ok(weight, value) or tuple(weight.shape) != (value.shape[-1],)):
            return False
        if backward:
            gradient, statistics = arrays[2:]
            rows = value.numel() // value.shape[-1]
            return (self._ok(gradient, value) and gradient.shape == value.shape and isinstance(statistics, torch.Tensor)
                    and statistics.dtype == torch.float32 and statistics.device == value.device
                    and statistics.is_contiguous() and tuple(statistics.shape) == (rows, 2))
        bias = arrays[2]
        return bias is None or (name == "layer_norm" and self._ok(bias, value)
                                and tuple(bias.shape) == (value.shape[-1],))

    def run(self, operation, arrays, *, eps=None, save_stats=True, needs=(True, True, True)):
        """namitorch/backends/cuda/normalization.py:182-235."""
        if not self.supports(operation, arrays):
            return None
        backward = operation.endswith("_backward")
        name = operation.removesuffix("_backward")
        if backward:
            if not isinstance(needs, tuple) or len(needs) != 3 or any(type(flag) is not bool for flag in needs):
                raise TypeError("Normalization gradient requirements must be three Python bools.")
            return self._backward(name, arrays, needs)
        if type(save_stats) is not bool:
            raise TypeError("save_stats must be a Python bool.")
        if (isinstance(eps, (bool, np.bool_)) or not isinstance(eps, (float, int, np.floating))
                or not math.isfinite(eps) or not 0 < eps <= float(np.finfo(np.float32).max)):
            raise ValueError("Normalization eps must be positive and finite in float32.")
        with np.errstate(under="ignore"):
            epsilon = np.float32(eps)
        if epsilon == 0:
            raise ValueError("Normalization eps must remain positive in float32.")
        value, weight, bias = arrays
        width = value.shape[-1]
        rows = value.numel() // width
        output = torch.empty_like(value)
        statistics = torch.empty((rows, 2), dtype=torch.float32, device=value.device) if save_stats else None
        if rows:
            args = N.NormArgs(op=N.NORM_OPS[name], dtype=N.dtype_code(value.dtype), input=value.data_ptr(),
                              weight=None if weight is None else weight.data_ptr(),
                              bias=None if bias is None else bias.data_ptr(), output=output.data_ptr(),
                              statistics=None if statistics is None else statistics.data_ptr(), rows=rows,
                              width=width, eps=float(epsilon))
            with torch.cuda.device(value.device):
                N.call("nt_norm_forward", N.C.byref(args), N.stream_handle())
        return output, statistics

    def _backward(self, name, arrays, needs):
        value, weight, gradient, statistics = arrays
        width = value.shape[-1]
        rows = value.numel() // width
        dx = torch.empty_like(value) if needs[0] else None
        dw = torch.empty(width, dtype=torch.float32, device=value.device) if needs[1] else None
        db = torch.empty(width, dtype=torch.float32, device=value.device) if needs[2] else None
        workspace = None
        if (needs[1] or needs[2]) and rows:
            size = int(N.load().nt_norm_workspace_size(rows, width))
            workspace = torch.empty(size, dtype=torch.uint8, device=value.device)
        args = N.NormArgs(op=N.NORM_OPS[name], dtype=N.dtype_code(value.dtype), input=value.data_ptr(),
                          weight=None if weight is None else weight.data_ptr(), gradient=gradient.data_ptr(),
                          statistics=statistics.data_ptr(), grad_input=None if dx is None else dx.data_ptr(),
                          grad_weight=None if dw is None else dw.data_ptr(),
                          grad_bias=None if db is None else db.data_ptr(),
                          workspace=None if workspace is None else workspace.data_ptr(),
                          workspace_bytes=0 if workspace is None else workspace.numel(), rows=rows, width=width)
        with torch.cuda.device(value.device):
            N.call("nt_norm_backward", N.C.byref(args), N.stream_handle(),
                   launches=int(rows > 0 and (dx is not None or workspace is not None)) + int(workspace is not None))
        cast = (lambda t: t if t is None or t.dtype == value.dtype else t.to(value.dtype))
        return dx, cast(dw), cast(db)


__all__ = ["NormalizationCUDAKernels"]
