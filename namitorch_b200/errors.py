"""Exception classes of the reference's CUDA backend, kept with the same names and fields."""
from __future__ import annotations

import re


class NamiTorchCUDAOutOfMemoryError(MemoryError):
    """Device allocation failure (namitorch/backends/_cuda_memory.py:8-21)."""

    def __init__(self, device, requested_bytes, allocated_bytes, reserved_bytes, free_bytes, total_bytes):
        self.device = device
        self.requested_bytes = requested_bytes
        self.allocated_bytes = allocated_bytes
        self.reserved_bytes = reserved_bytes
        self.free_bytes = free_bytes
        self.total_bytes = total_bytes
        fields = (("requested", requested_bytes), ("allocated", allocated_bytes), ("reserved", reserved_bytes),
                  ("free", free_bytes), ("total", total_bytes))
        details = ", ".join(f"{name}={value} bytes" if value is not None else f"{name}=unavailable"
                            for name, value in fields)
        super().__init__(f"NamiTorch CUDA out of memory on {device}: {details}.")

    @classmethod
    def from_message(cls, message: str) -> "NamiTorchCUDAOutOfMemoryError":
        def field(name):
            m = re.search(rf"{name}=(\d+)", message)
            return int(m.group(1)) if m else None

        m = re.search(r"cuda:(\d+)", message)
        device = f"cuda:{m.group(1)}" if m else "cuda"
        return cls(device, field("requested"), None, None, field("free"), field("total"))


class CUDAKernelCompilationError(RuntimeError):
    """Raised when the sm_100a library cannot be built (namitorch/backends/cuda/kernels.py:150-161)."""


class NativeLibraryError(RuntimeError):
    """The compiled library is missing or does not match this package."""
