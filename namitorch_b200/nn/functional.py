"""Fused softmax cross-entropy (namitorch/nn/functional.py:792-863).

``cross_entropy`` keeps the reference signature and validation. One kernel launch
(``nt_softmax_xent``) reads the logits once and produces both the loss and, when the logits
require grad, the gradient for a unit upstream gradient; the autograd backward only scales
it by the incoming gradient (and skips even that when the incoming gradient is exactly 1).
float16 / bfloat16 logits are read directly and reduced in float32 — the reference promotes
them to float32 first (``float32_function``) — and the gradient comes back in the logits'
dtype. ``softmax_cross_entropy`` exposes the fused forward + backward without autograd.
"""
from __future__ import annotations

from numbers import Integral, Real

import numpy as np
import torch

from .. import _native as N
from ..flat import xent_workspace

_REDUCTIONS = {"none": N.NT_REDUCTION_NONE, "mean": N.NT_REDUCTION_MEAN, "sum": N.NT_REDUCTION_SUM}


def _label_smoothing(value) -> float:
    if isinstance(value, (bool, np.bool_)) or not isinstance(value, Real):
        raise TypeError("label_smoothing must be a real scalar.")
    epsilon = float(value)
    if not 0 <= epsilon < 1:
        raise ValueError("label_smoothing must be in [0, 1).")
    return epsilon


def _arguments(input, target, weight, ignore_index, reduction):
    """namitorch/nn/functional.py:792-816 (the range check runs on the device)."""
    if reduction not in _REDUCTIONS:
        raise ValueError(f"Unsupported loss reduction {reduction!r}; expected 'none', 'mean' or 'sum'.")
    if not isinstance(input, torch.Tensor):
        raise TypeError("Loss input must be a NamiTorch Tensor.")
    if not input.dtype.is_floating_point:
        raise TypeError("Classification loss input must be a floating Tensor.")
    if input.ndim < 1 or input.shape[-1] == 0:
        raise ValueError(f"Classification loss input must have shape [..., C] with C > 0, got {tuple(input.shape)}.")
    if not isinstance(target, torch.Tensor) or target.dtype.is_floating_point or target.dtype == torch.bool:
        raise TypeError("Classification loss target must be an integer Tensor.")
    if tuple(target.shape) != tuple(input.shape[:-1]):
        raise ValueError(f"Target shape {tuple(target.shape)} must equal input shape without the last class axis "
                         f"{tuple(input.shape[:-1])}.")
    if isinstance(ignore_index, (bool, np.bool_)) or not isinstance(ignore_index, Integral):
        raise TypeError("ignore_index must be an integer.")
    classes = input.shape[-1]
    if weight is not None:
        if not isinstance(weight, torch.Tensor) or not weight.dtype.is_floating_point:
            raise TypeError("Class weight must be a floating Tensor.")
        if weight.ndim != 1 or weight.shape[0] == 0:
            raise ValueError(f"Class weight must have shape [C] with C > 0, got {tuple(weight.shape)}.")
        if weight.shape != (classes,):
            raise ValueError(f"Class weight must have shape {(classes,)}, got {tuple(weight.shape)}.")
    if input.device.type != "cuda" or target.device != input.device or (weight is not None and weight.device != input.device):
        raise RuntimeError("namitorch_b200 cross_entropy runs on one CUDA device; move logits, targets and weights "
                           "there first.")
    if input.dtype not in (torch.float32, torch.float16, torch.bfloat16):
        raise TypeError(f"cross_entropy supports float32, float16 and bfloat16 logits, got {input.dtype}.")
    logits = input.reshape(-1, classes)
    if not logits.is_contiguous():
        logits = logits.contiguous()
    targets = target.reshape(-1).to(torch.int64).contiguous()
    w = None if weight is None else weight.to(torch.float32).contiguous()
    return logits, targets, w, int(ignore_index), _REDUCTIONS[reduction]


def _launch(logits, targets, weight, ignore_index, reduction, smoothing, want_grad):
    rows, classes = logits.shape
    device = logits.device
    with torch.cuda.device(device):
        loss = torch.empty(rows if reduction == N.NT_REDUCTION_NONE else 1, dtype=torch.float32, device=device)
        row_loss = loss if reduction == N.NT_REDUCTION_NONE else torch.empty(max(rows, 1), dtype=torch.float32,
                                                                             device=device)
        dlogits = torch.empty_like(logits) if want_grad else None
        info = torch.empty(len(N.XENT_INFO_FIELDS), dtype=torch.float64, device=device)   # reset by the call
        ws = xent_workspace(device)
        args = N.XentArgs(
            logits=logits.data_ptr() if rows else None, dtype=N.dtype_code(logits.dtype), rows=rows, classes=classes,
            targets=targets.data_ptr() if rows else None, ignore_index=ignore_index,
            class_weight=None if weight is None else weight.data_ptr(), label_smoothing=float(smoothing),
            reduction=reduction, dlogits=None if dlogits is None or rows == 0 else dlogits.data_ptr(),
            loss=loss.data_ptr(), row_loss=row_loss.data_ptr(), info=info.data_ptr(), workspace=ws.data_ptr(),
            workspace_bytes=ws.numel())
        # One kernel (with a memset of the info record) without class weights; the one-block
        # prepare kernel first with them, or alone for zero rows.
        N.call("nt_softmax_xent", N.C.byref(args), N.stream_handle(),
               launches=(1 if rows else 0) + (0 if weight is None and rows else 1))
    return loss, dlogits, info


def _validate_targets(info: torch.Tensor, classes: int) -> None:
    bad = float(info[N.XENT_INFO_FIELDS.index("bad_targets")].item())
    if bad:
        raise IndexError(f"Every non-ignored target must be in [0, {classes}).")


def softmax_cross_entropy(logits: torch.Tensor, target: torch.Tensor, weight: torch.Tensor | None = None,
                          ignore_index: int = -100, reduction: str = "mean", label_smoothing: float = 0.0,
                          *, validate: bool = True):
    """Fused forward + backward: returns (loss, dlogits) for a unit upstream gradient.

    ``validate=False`` skips the host read that turns out-of-range targets into IndexError
    (those rows then count as ignored)."""
    epsilon = _label_smoothing(label_smoothing)
    x, t, w, ignore, red = _arguments(logits, target, weight, ignore_index, reduction)
    loss, dlogits, info = _launch(x, t, w, ignore, red, epsilon, True)
    if validate:
        _validate_targets(info, x.shape[1])
    out = loss.reshape(target.shape) if red == N.NT_REDUCTION_NONE else loss[0]
    return out, dlogits.reshape(logits.shape)


class _CrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, target, weight, ignore_index, reduction, epsilon, validate):
        want_grad = ctx.needs_input_grad[0]
        loss, dlogits, info = _launch(logits, target, weight, ignore_index, reduction, epsilon, want_grad)
        if validate:
            _validate_targets(info, logits.shape[1])
        ctx.reduction = reduction
        ctx.used = False
        if want_grad:
            ctx.save_for_backward(dlogits)
        return loss if reduction == N.NT_REDUCTION_NONE else loss[0]

    @staticmethod
    def backward(ctx, grad_output):
        # The gradient was computed by the forward launch; it is scaled in place, once.
        if ctx.used:
            raise RuntimeError("The fused cross_entropy gradient can be taken once per forward call.")
        ctx.used = True
        (dlogits,) = ctx.saved_tensors
        rows, classes = dlogits.shape
        g = grad_output.to(torch.float32).contiguous()
        with torch.cuda.device(dlogits.device):
            N.call("nt_xent_backward_scale", dlogits.data_ptr(), N.dtype_code(dlogits.dtype), rows, classes,
                   g.data_ptr(), int(ctx.reduction == N.NT_REDUCTION_NONE), N.stream_handle())
        return dlogits, None, None, None, None, None, None


def cross_entropy(input: torch.Tensor, target: torch.Tensor, weight: torch.Tensor | None = None,
                  ignore_index: int = -100, reduction: str = "mean", label_smoothing: float = 0.0) -> torch.Tensor:
    """namitorch/nn/functional.py:856-863."""
    epsilon = _label_smoothing(label_smoothing)
    x, t, w, ignore, red = _arguments(input, target, weight, ignore_index, reduction)
    loss = _CrossEntropy.apply(x, t, w, ignore, red, epsilon, True)
    return loss.reshape(target.shape) if red == N.NT_REDUCTION_NONE else loss


def linear(input: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """``input @ weight.T + bias`` with the reference's checks and autocast rule
    (namitorch/nn/functional.py:44-65): inside an enabled autocast context the operands are
    converted to the autocast dtype (``amp.autocast_operands``), which for parameters held in
    an optimizer's ``model_dtype`` copy is no conversion at all. Operands of different dtypes
    outside autocast are promoted, as the reference's matmul promotes them. The product is a
    library GEMM (torch / cuBLAS); it is not part of this package's kernels."""
    from ..amp import autocast_operands
    if not isinstance(input, torch.Tensor) or not isinstance(weight, torch.Tensor):
        raise TypeError("linear input and weight must be NamiTorch Tensors.")
    if weight.ndim != 2:
        raise ValueError(f"linear weight must have rank 2, got shape {tuple(weight.shape)}.")
    if input.ndim < 1 or input.shape[-1] != weight.shape[1]:
        raise ValueError(f"linear input must have rank >= 1 and last dimension {weight.shape[1]}, got shape "
                         f"{tuple(input.shape)}.")
    if bias is not None:
        if not isinstance(bias, torch.Tensor):
            raise TypeError("linear bias must be a NamiTorch Tensor or None.")
        if tuple(bias.shape) != (weight.shape[0],):
            raise ValueError(f"linear bias must have shape {(weight.shape[0],)}, got {tuple(bias.shape)}.")
    if weight.device != input.device or (bias is not None and bias.device != input.device):
        raise RuntimeError("linear operands must be on the same device.")
    input, weight, bias = autocast_operands("linear", input, weight, bias)
    common = torch.promote_types(input.dtype, weight.dtype)
    if bias is not None:
        common = torch.promote_types(common, bias.dtype)
    input, weight = input.to(common), weight.to(common)
    bias = None if bias is None else bias.to(common)
    return torch.nn.functional.linear(input, weight, bias)


__all__ = ["cross_entropy", "linear", "softmax_cross_entropy"]
