"""The fused elementwise plugin seam (namitorch/backends/cuda/fused.py:88-133) on torch tensors.

``FusedCUDAKernels.supports(operation, arrays)`` and ``run(operation, arrays)`` keep the
reference's operations, operand layouts and shape rules: ``run`` returns None when the
arrays are not supported (the caller then takes its own path), one new tensor otherwise, and
a pair for ``swiglu_backward``. Operand layouts (the reference's names):

- unary ``(x,)``: sigmoid, silu, gelu_tanh
- unary_backward ``(saved, grad)``: sigmoid_backward (saved = sigmoid output),
  silu_backward, gelu_tanh_backward (saved = input)
- pair ``(gate, up)``: swiglu; pair_backward ``(gate, up, grad)``: swiglu_backward
- bias ``(x, bias[width])``: bias_{sigmoid,silu,gelu_tanh,relu}; bias_backward
  ``(x, bias, grad)``: the same with ``_backward``, the elementwise local gradient
- clamp ``(x, min or None, max or None)`` with 0-d bounds; clamp_backward adds ``grad``.

The kernel is ``nt_fused_elementwise``. Besides float32 (the reference's only dtype) it
takes float16 and bfloat16 operands, computed in float32.
"""
from __future__ import annotations

import torch

from .. import _native as N

_LAYOUTS = {
    "sigmoid": "unary", "silu": "unary", "gelu_tanh": "unary",
    "sigmoid_backward": "unary_backward", "silu_backward": "unary_backward", "gelu_tanh_backward": "unary_backward",
    "swiglu": "pair", "swiglu_backward": "pair_backward",
    "clamp": "clamp", "clamp_backward": "clamp_backward",
}
for _name in ("sigmoid", "silu", "gelu_tanh", "relu"):
    _LAYOUTS[f"bias_{_name}"] = "bias"
    _LAYOUTS[f"bias_{_name}_backward"] = "bias_backward"
del _name
_ARITY = {"unary": 1, "unary_backward": 2, "pair": 2, "pair_backward": 3, "bias": 2, "bias_backward": 3,
          "clamp": 3, "clamp_backward": 4}
_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
OPERATIONS = frozenset(_LAYOUTS)


class FusedCUDAKernels:
    def __init__(self, backend=None):
        self._backend = backend

    def supports(self, operation, arrays) -> bool:
        """namitorch/backends/cuda/fused.py:89-113."""
        layout = _LAYOUTS.get(operation)
        if layout is None or len(arrays) != _ARITY[layout] or arrays[0] is None:
            return False
        first = arrays[0]
        for position, array in enumerate(arrays):
            if array is None:
                if not layout.startswith("clamp") or position not in (1, 2):
                    return False
                continue
            if not isinstance(array, torch.Tensor) or array.device.type != "cuda" or array.device != first.device:
                return False
            if array.dtype not in _DTYPES or array.dtype != first.dtype or not array.is_contiguous():
                return False
            if array.data_ptr() % array.element_size():
                return False
        if layout.startswith("bias"):
            return first.dim() >= 1 and tuple(arrays[1].shape) == (first.shape[-1],) and (
                len(arrays) == 2 or arrays[2].shape == first.shape)
        if layout.startswith("clamp"):
            bounds = arrays[1:3]
            return any(b is not None for b in bounds) and all(b is None or b.dim() == 0 for b in bounds) and (
                len(arrays) == 3 or arrays[3].shape == first.shape)
        return all(array.shape == first.shape for array in arrays[1:])

    def run(self, operation, arrays):
        """namitorch/backends/cuda/fused.py:115-133."""
        if not self.supports(operation, arrays):
            return None
        first = arrays[0]
        layout = _LAYOUTS[operation]
        outputs = tuple(torch.empty_like(first) for _ in range(2 if operation == "swiglu_backward" else 1))
        count = first.numel()
        if count:
            ptr = (lambda t: None if t is None else t.data_ptr())
            args = N.FusedArgs(op=N.FUSED_OPS[operation], dtype=N.dtype_code(first.dtype), a=first.data_ptr(),
                               b=ptr(arrays[1]) if len(arrays) > 1 else None,
                               c=ptr(arrays[2]) if len(arrays) > 2 else None,
                               d=ptr(arrays[3]) if len(arrays) > 3 else None,
                               output=outputs[0].data_ptr(), second=outputs[-1].data_ptr() if len(outputs) == 2 else None,
                               count=count, width=first.shape[-1] if layout.startswith("bias") else 1)
            with torch.cuda.device(first.device):
                N.call("nt_fused_elementwise", N.C.byref(args), N.stream_handle())
        return outputs if len(outputs) == 2 else outputs[0]


__all__ = ["FusedCUDAKernels", "OPERATIONS"]
