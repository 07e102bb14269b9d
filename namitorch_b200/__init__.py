"""namitorch_b200 — B200 (sm_100a) implementation of NamiTorch's optimizer-step and
mixed-precision hot path.

Public modules mirror the reference's: ``optim`` (Adam, AdamW, clip_grad_norm_, ...),
``amp`` (autocast, GradScaler), ``nn.functional`` (cross_entropy) and ``backends``
(enable_fused_kernels, the ``backend.adamw`` seam), plus ``zero`` (ZeRO-1 sharded AdamW
across GPUs). All compute runs in ``lib/libnamitorch_b200.so``; see include/namitorch_b200.h.
"""
from . import amp, backends, nn, optim, workloads
from ._native import load as load_library
from .amp import GradScaler, autocast
from .backends import enable_fused_kernels
from .errors import CUDAKernelCompilationError, NamiTorchCUDAOutOfMemoryError, NativeLibraryError

__version__ = "0.1.0"

__all__ = ["amp", "backends", "nn", "optim", "workloads", "GradScaler", "autocast", "enable_fused_kernels",
           "load_library", "NamiTorchCUDAOutOfMemoryError", "CUDAKernelCompilationError", "NativeLibraryError"]
