"""The row-softmax plugin seam (namitorch/backends/cuda/softmax.py:110-178) on torch tensors.

``SoftmaxCUDAKernels.supports(operation, arrays)`` and ``run(operation, arrays, *,
query_position_offset=0, require_nonempty=False)`` keep the reference's operations, argument
checks and errors: ``run`` returns None when the arrays are not supported (the caller then
takes its own path), raises ValueError for a masked attention row that is empty or holds NaN
/ +inf when ``require_nonempty`` is set. The kernel is ``nt_row_softmax``. Besides float32
(the reference's only dtype) it takes float16 and bfloat16 rows, computed in float32.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _native as N

OPERATIONS = frozenset(N.SOFTMAX_OPS)
_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def mask_rows(mask_shape, shape):
    """Rows of a mask broadcast against `shape` (namitorch/backends/cuda/softmax.py:91-107):
    0 for one row shared by all, None when the mask does not broadcast as whole rows."""
    mask_shape, shape = tuple(mask_shape), tuple(shape)
    if len(mask_shape) > len(shape):
        return None
    padded = (1,) * (len(shape) - len(mask_shape)) + mask_shape
    if any(a != 1 and a != b for a, b in zip(padded, shape)):
        return None
    if all(n == 1 for n in padded):
        return 0
    if padded[-1] != shape[-1]:
        return None
    first = next(i for i, n in enumerate(padded) if n != 1)
    if padded[first:] != shape[first:]:
        return None
    rows = 1
    for n in padded[:-1]:
        rows *= n
    return rows


class SoftmaxCUDAKernels:
    def __init__(self, backend=None):
        self._backend = backend

    def supports(self, operation, arrays) -> bool:
        """namitorch/backends/cuda/softmax.py:111-135."""
        if operation not in OPERATIONS or not arrays:
            return False
        backward = operation.endswith("_backward")
        masked = operation.startswith(("masked", "causal"))
        if len(arrays) != 1 + int(backward) + int(masked):
            return False
        value = arrays[0]
        for array in arrays[:2 if backward else 1]:
            if not isinstance(array, torch.Tensor) or array.device.type != "cuda" or array.device != value.device:
                return False
            if array.dtype not in _DTYPES or array.dtype != value.dtype or not array.is_contiguous():
                return False
            if array.data_ptr() % array.element_size() or array.shape != value.shape:
                return False
        if value.dim() == 0 or value.shape[-1] > N.NT_SOFTMAX_MAX_WIDTH:
            return False
        if operation.startswith("causal") and value.dim() < 2:
            return False
        if masked:
            mask = arrays[-1]
            if mask is None:
                return operation.startswith("causal")
            if not isinstance(mask, torch.Tensor) or mask.device != value.device:
                return False
            if mask.dtype != torch.bool or not mask.is_contiguous() or mask_rows(mask.shape, value.shape) is None:
                return False
        return True

    def run(self, operation, arrays, *, query_position_offset=0, require_nonempty=False):
        """namitorch/backends/cuda/softmax.py:137-178."""
        if not self.supports(operation, arrays):
            return None
        if type(query_position_offset) is not int or query_position_offset < 0:
            raise ValueError("query_position_offset must be a nonnegative Python integer.")
        if type(require_nonempty) is not bool:
            raise TypeError("require_nonempty must be a Python bool.")
        value = arrays[0]
        backward = operation.endswith("_backward")
        masked = operation.startswith(("masked", "causal"))
        mask = arrays[-1] if masked else None
        width = value.shape[-1]
        rows = value.numel() // width if width else 0
        output = torch.empty_like(value)
        if not rows:
            return output
        summary = None
        if require_nonempty and not backward:
            summary = torch.tensor([0, 0, -1, 0], dtype=torch.int64, device=value.device)
        args = N.SoftmaxArgs(
            op=N.SOFTMAX_OPS[operation], dtype=N.dtype_code(value.dtype), input=value.data_ptr(),
            gradient=arrays[1].data_ptr() if backward else None,
            mask=None if mask is None else mask.data_ptr(), output=output.data_ptr(),
            summary=None if summary is None else summary.data_ptr(), rows=rows, width=width,
            mask_rows=0 if mask is None else mask_rows(mask.shape, value.shape),
            queries=max(1, value.shape[-2]) if value.dim() > 1 else 1, offset=min(query_position_offset, width))
        with torch.cuda.device(value.device):
            N.call("nt_row_softmax", N.C.byref(args), N.stream_handle())
        if summary is not None:
            empty, invalid, first, _ = summary.tolist()
            if invalid:
                raise ValueError("Masked attention scores must be finite or -inf.")
            if empty:
                coordinate = tuple(int(i) for i in np.unravel_index(first, tuple(value.shape[:-1])))
                raise ValueError(f"Attention row {coordinate} has no allowed keys.")
        return output


__all__ = ["SoftmaxCUDAKernels", "mask_rows", "OPERATIONS"]
