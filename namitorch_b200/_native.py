"""ctypes binding of ``libnamitorch_b200.so`` (declared in include/namitorch_b200.h).

This module is the only place that touches the C ABI. It mirrors the header's structs,
maps status codes to the reference's exception classes and passes CUDA streams as raw
handles. There is no fallback: if the library cannot be loaded, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading
from pathlib import Path

from .errors import NamiTorchCUDAOutOfMemoryError, NativeLibraryError

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libnamitorch_b200.so"

NT_OK, NT_EINVAL, NT_ECUDA, NT_ENOMEM, NT_EUNSUPPORTED = 0, 1, 2, 3, 4
NT_F32, NT_F16, NT_BF16 = 0, 1, 2
NT_REDUCTION_NONE, NT_REDUCTION_MEAN, NT_REDUCTION_SUM = 0, 1, 2
NT_DECAY_NONE, NT_DECAY_DECOUPLED, NT_DECAY_COUPLED = 0, 1, 2
NT_MAX_GROUPS = 32
NT_MAX_FOUND_INF = 16
NT_MAX_RANKS = 8
ABI_VERSION = 8


class Segment(C.Structure):
    _fields_ = [("grad", C.c_void_p), ("offset", C.c_int64), ("count", C.c_int64), ("chunk_begin", C.c_int64),
                ("group", C.c_int32), ("step_slot", C.c_int32)]


class AdamWGroup(C.Structure):
    _fields_ = [("lr", C.c_float), ("beta1", C.c_float), ("beta2", C.c_float), ("one_minus_beta1", C.c_float),
                ("one_minus_beta2", C.c_float), ("eps", C.c_float), ("weight_decay", C.c_float),
                ("decay_factor", C.c_float), ("maximize", C.c_int32), ("decay_mode", C.c_int32),
                ("update_parameter", C.c_int32), ("correction_row", C.c_int32), ("schedule_column", C.c_int32),
                ("reserved", C.c_int32)]


class LrEntry(C.Structure):
    _fields_ = [("lr", C.c_float), ("decay_factor", C.c_float), ("update_parameter", C.c_int32),
                ("reserved", C.c_int32)]


class Stats(C.Structure):
    _fields_ = [("sumsq", C.c_double), ("nonfinite", C.c_double), ("nan", C.c_double), ("maxabs", C.c_double),
                ("powsum", C.c_double), ("norm", C.c_double), ("found_inf", C.c_double), ("error", C.c_double)]


STATS_FIELDS = [name for name, _ in Stats._fields_]
STATS_DOUBLES = len(STATS_FIELDS)


class AdamWMtArgs(C.Structure):
    _fields_ = [("param", C.c_void_p), ("exp_avg", C.c_void_p), ("exp_avg_sq", C.c_void_p),
                ("model_copy", C.c_void_p), ("model_dtype", C.c_int32), ("grad_dtype", C.c_int32),
                ("segments", C.c_void_p), ("num_segments", C.c_int32), ("chunk_elems", C.c_int32),
                ("num_chunks", C.c_int64), ("steps", C.c_void_p), ("corrections", C.c_void_p),
                ("correction_capacity", C.c_int32), ("scale", C.c_void_p), ("stats", C.c_void_p),
                ("skip_nonfinite", C.c_int32), ("clip", C.c_int32), ("max_norm", C.c_double),
                ("workspace", C.c_void_p), ("error", C.c_void_p), ("groups", C.POINTER(AdamWGroup)),
                ("num_groups", C.c_int32), ("lr_schedule", C.c_void_p), ("lr_schedule_rows", C.c_int32),
                ("lr_schedule_columns", C.c_int32), ("lr_step", C.c_void_p)]


class Span(C.Structure):
    _fields_ = [("ptr", C.c_void_p), ("count", C.c_int64), ("chunk_begin", C.c_int64)]


class GradStatsArgs(C.Structure):
    _fields_ = [("spans", C.c_void_p), ("num_spans", C.c_int32), ("chunk_elems", C.c_int32),
                ("num_chunks", C.c_int64), ("dtype", C.c_int32), ("scale", C.c_void_p), ("pass_", C.c_int32),
                ("norm_type", C.c_double), ("finalize", C.c_int32), ("stats", C.c_void_p),
                ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t)]


class XentInfo(C.Structure):
    _fields_ = [("denominator", C.c_double), ("weight_sum", C.c_double), ("loss_sum", C.c_double),
                ("n_valid", C.c_double), ("bad_targets", C.c_double), ("error", C.c_double),
                ("reserved0", C.c_double), ("reserved1", C.c_double)]


XENT_INFO_FIELDS = [name for name, _ in XentInfo._fields_]


class XentArgs(C.Structure):
    _fields_ = [("logits", C.c_void_p), ("dtype", C.c_int32), ("rows", C.c_int64), ("classes", C.c_int64),
                ("targets", C.c_void_p), ("ignore_index", C.c_int64), ("class_weight", C.c_void_p),
                ("label_smoothing", C.c_float), ("reduction", C.c_int32), ("dlogits", C.c_void_p),
                ("loss", C.c_void_p), ("row_loss", C.c_void_p), ("info", C.c_void_p), ("workspace", C.c_void_p),
                ("workspace_bytes", C.c_size_t)]


NT_SOFTMAX_MAX_WIDTH = 4096
SOFTMAX_OPS = {"softmax": 0, "masked_softmax": 1, "causal_softmax": 2, "softmax_backward": 3,
               "masked_softmax_backward": 4, "causal_softmax_backward": 5}


class SoftmaxArgs(C.Structure):
    _fields_ = [("op", C.c_int32), ("dtype", C.c_int32), ("input", C.c_void_p), ("gradient", C.c_void_p),
                ("mask", C.c_void_p), ("output", C.c_void_p), ("summary", C.c_void_p), ("rows", C.c_int64),
                ("width", C.c_int64), ("mask_rows", C.c_int64), ("queries", C.c_int64), ("offset", C.c_int64)]


NT_NORM_MAX_WIDTH = 8192
NORM_OPS = {"rms_norm": 0, "layer_norm": 1}

FUSED_OPS = {"sigmoid": 0, "silu": 1, "gelu_tanh": 2, "sigmoid_backward": 3, "silu_backward": 4,
             "gelu_tanh_backward": 5, "swiglu": 6, "swiglu_backward": 7, "bias_sigmoid": 8, "bias_silu": 9,
             "bias_gelu_tanh": 10, "bias_relu": 11, "bias_sigmoid_backward": 12, "bias_silu_backward": 13,
             "bias_gelu_tanh_backward": 14, "bias_relu_backward": 15, "clamp": 16, "clamp_backward": 17}


class FusedArgs(C.Structure):
    _fields_ = [("op", C.c_int32), ("dtype", C.c_int32), ("a", C.c_void_p), ("b", C.c_void_p), ("c", C.c_void_p),
                ("d", C.c_void_p), ("output", C.c_void_p), ("second", C.c_void_p), ("count", C.c_int64),
                ("width", C.c_int64)]


class NormArgs(C.Structure):
    _fields_ = [("op", C.c_int32), ("dtype", C.c_int32), ("input", C.c_void_p), ("weight", C.c_void_p),
                ("bias", C.c_void_p), ("output", C.c_void_p), ("statistics", C.c_void_p), ("gradient", C.c_void_p),
                ("grad_input", C.c_void_p), ("grad_weight", C.c_void_p), ("grad_bias", C.c_void_p),
                ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t), ("rows", C.c_int64),
                ("width", C.c_int64), ("eps", C.c_float)]


class ZeroReduceArgs(C.Structure):
    _fields_ = [("sources", C.c_void_p * NT_MAX_RANKS), ("num_ranks", C.c_int32), ("dtype", C.c_int32),
                ("count", C.c_int64), ("average", C.c_int32), ("dest", C.c_void_p), ("scale", C.c_void_p),
                ("stats", C.c_void_p), ("workspace", C.c_void_p), ("workspace_bytes", C.c_size_t)]


NT_ZERO_READY, NT_ZERO_STATS, NT_ZERO_DONE = 0, 1, 2


class ZeroMailbox(C.Structure):
    _fields_ = [("flags", (C.c_uint64 * NT_MAX_RANKS) * 3), ("stats", (C.c_double * 4) * NT_MAX_RANKS)]


class ZeroSync(C.Structure):
    _fields_ = [("mailboxes", C.c_void_p * NT_MAX_RANKS), ("rank", C.c_int32), ("reserved", C.c_int32),
                ("epoch", C.c_uint64), ("timeout_ns", C.c_uint64), ("error", C.c_void_p)]


# name -> (restype, argtypes). Every symbol of include/namitorch_b200.h.
SIGNATURES: dict[str, tuple] = {
    "nt_abi_version": (C.c_int, []),
    "nt_last_error": (C.c_char_p, []),
    "nt_device_init": (C.c_int, [C.c_int]),
    "nt_sm_count": (C.c_int, [C.POINTER(C.c_int)]),
    "nt_malloc": (C.c_int, [C.POINTER(C.c_void_p), C.c_size_t]),
    "nt_free": (C.c_int, [C.c_void_p]),
    "nt_mem_info": (C.c_int, [C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    "nt_memset_async": (C.c_int, [C.c_void_p, C.c_int, C.c_size_t, C.c_void_p]),
    "nt_memcpy_async": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "nt_memcpy_sync": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t]),
    "nt_stream_synchronize": (C.c_int, [C.c_void_p]),
    "nt_cast": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int64, C.c_void_p]),
    "nt_adamw_f32": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.POINTER(C.c_float), C.c_int,
                               C.c_int, C.c_uint64, C.c_void_p]),
    "nt_adamw_workspace_size": (C.c_size_t, []),
    "nt_adamw_mt": (C.c_int, [C.POINTER(AdamWMtArgs), C.c_void_p]),
    "nt_grad_stats_workspace_size": (C.c_size_t, []),
    "nt_grad_stats": (C.c_int, [C.POINTER(GradStatsArgs), C.c_void_p]),
    "nt_grad_stats_finalize": (C.c_int, [C.c_void_p, C.c_double, C.c_void_p]),
    "nt_schedule_step": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p), C.c_int32, C.c_void_p]),
    "nt_grad_stats_noalloc_scratch_bytes": (C.c_size_t, []),
    "nt_grad_stats_noalloc": (C.c_int, [C.POINTER(Span), C.c_int32, C.c_int32, C.c_void_p, C.c_double,
                                        C.c_void_p, C.c_void_p]),
    "nt_grad_transform": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int64, C.c_int32, C.c_void_p,
                                    C.c_void_p, C.c_int32, C.c_double, C.c_void_p]),
    "nt_grad_clip_value": (C.c_int, [C.c_void_p, C.c_int32, C.c_int32, C.c_int64, C.c_int32, C.c_double,
                                     C.c_void_p]),
    "nt_scaler_update": (C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p), C.c_int32, C.c_double,
                                   C.c_double, C.c_int32, C.c_void_p]),
    "nt_ipc_export": (C.c_int, [C.c_void_p, C.POINTER(C.c_ubyte), C.POINTER(C.c_uint64)]),
    "nt_ipc_open": (C.c_int, [C.POINTER(C.c_ubyte), C.c_uint64, C.POINTER(C.c_void_p)]),
    "nt_ipc_close": (C.c_int, [C.c_void_p]),
    "nt_can_access_peer": (C.c_int, [C.c_int32, C.POINTER(C.c_int32)]),
    "nt_zero_reduce_scatter_stats": (C.c_int, [C.POINTER(ZeroReduceArgs), C.c_void_p]),
    "nt_adamw_mt_push": (C.c_int, [C.POINTER(AdamWMtArgs), C.POINTER(C.c_void_p), C.c_int32, C.c_void_p]),
    "nt_peer_copy": (C.c_int, [C.POINTER(C.c_void_p), C.POINTER(C.c_void_p), C.c_int32, C.c_uint64, C.c_void_p]),
    "nt_zero_flag_exchange": (C.c_int, [C.POINTER(ZeroSync), C.c_int32, C.c_int32, C.c_void_p, C.c_void_p]),
    "nt_zero_stats_exchange": (C.c_int, [C.c_void_p, C.c_int32, C.POINTER(ZeroSync), C.c_int32, C.c_void_p,
                                         C.c_double, C.c_void_p, C.c_void_p]),
    "nt_zero_reduce_scatter_exchange": (C.c_int, [C.POINTER(ZeroReduceArgs), C.POINTER(ZeroSync), C.c_double,
                                                   C.c_void_p]),
    "nt_adamw_mt_push_exchange": (C.c_int, [C.POINTER(AdamWMtArgs), C.POINTER(C.c_void_p), C.c_int32,
                                            C.POINTER(ZeroSync), C.c_void_p]),
    "nt_row_softmax": (C.c_int, [C.POINTER(SoftmaxArgs), C.c_void_p]),
    "nt_norm_workspace_size": (C.c_size_t, [C.c_int64, C.c_int64]),
    "nt_norm_forward": (C.c_int, [C.POINTER(NormArgs), C.c_void_p]),
    "nt_norm_backward": (C.c_int, [C.POINTER(NormArgs), C.c_void_p]),
    "nt_fused_elementwise": (C.c_int, [C.POINTER(FusedArgs), C.c_void_p]),
    "nt_xent_workspace_size": (C.c_size_t, []),
    "nt_softmax_xent": (C.c_int, [C.POINTER(XentArgs), C.c_void_p]),
    "nt_xent_backward_scale": (C.c_int, [C.c_void_p, C.c_int32, C.c_int64, C.c_int64, C.c_void_p, C.c_int32,
                                         C.c_void_p]),
}

_lib = None
_lock = threading.Lock()


def load(path: str | os.PathLike | None = None):
    """Loads the shared library once and binds every declared symbol."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        target = Path(path) if path is not None else LIB_PATH
        if not target.exists():
            raise NativeLibraryError(
                f"{target} does not exist: build it with `python -m namitorch_b200._build` "
                "(namitorch_b200 has no CPU or Python fallback for its CUDA kernels).")
        try:
            lib = C.CDLL(str(target))
        except OSError as error:
            raise NativeLibraryError(f"cannot load {target}: {error}") from error
        for name, (restype, argtypes) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = restype
            fn.argtypes = argtypes
        if lib.nt_abi_version() != ABI_VERSION:
            raise NativeLibraryError(f"{target} has ABI {lib.nt_abi_version()}, expected {ABI_VERSION}")
        _lib = lib
        return lib


def last_error() -> str:
    return (load().nt_last_error() or b"").decode("utf-8", "replace")


def check(status: int, what: str = "") -> None:
    """Raises the exception class the reference uses for this kind of failure."""
    if status == NT_OK:
        return
    message = last_error() or what
    if status == NT_EINVAL:
        raise ValueError(message)
    if status == NT_ENOMEM:
        raise NamiTorchCUDAOutOfMemoryError.from_message(message)
    if status == NT_EUNSUPPORTED:
        raise RuntimeError(message)
    raise RuntimeError(f"CUDA error in {what or 'namitorch_b200'}: {message}")


# Kernel launches issued per successful call of each launching entry point (for the
# benchmark's launch count; the statistics entry point launches one kernel per call).
LAUNCHES_PER_CALL = {"nt_adamw_f32": 1, "nt_adamw_mt": 1, "nt_adamw_mt_push": 1, "nt_zero_reduce_scatter_stats": 1, "nt_peer_copy": 1,
                     "nt_zero_reduce_scatter_exchange": 1, "nt_adamw_mt_push_exchange": 1,
                     "nt_zero_flag_exchange": 1, "nt_zero_stats_exchange": 1,
                     "nt_grad_stats": 1, "nt_grad_stats_finalize": 1, "nt_schedule_step": 1, "nt_row_softmax": 1, "nt_norm_forward": 1,
                     "nt_grad_transform": 1, "nt_grad_clip_value": 1, "nt_scaler_update": 1,
                     "nt_softmax_xent": 2, "nt_xent_backward_scale": 1, "nt_cast": 1, "nt_fused_elementwise": 1}
launch_count = 0


def call(name: str, *args, launches: int | None = None) -> None:
    """Calls an entry point and raises on failure; counts the kernels it launched (the table
    above, or `launches` for entry points whose count depends on the arguments)."""
    global launch_count
    check(getattr(load(), name)(*args), name)
    launch_count += LAUNCHES_PER_CALL.get(name, 0) if launches is None else launches


def stream_handle(stream=None) -> int:
    """Raw cudaStream_t of a torch stream (default: the current stream of the current device)."""
    import torch
    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream)


def dtype_code(dtype) -> int:
    import torch
    codes = {torch.float32: NT_F32, torch.float16: NT_F16, torch.bfloat16: NT_BF16}
    if dtype not in codes:
        raise TypeError(f"namitorch_b200 kernels support float32, float16 and bfloat16, got {dtype}.")
    return codes[dtype]


def ipc_export(ptr: int) -> tuple[bytes, int]:
    """(CUDA IPC handle of the allocation holding ``ptr``, byte offset of ``ptr`` in it)."""
    handle = (C.c_ubyte * 64)()
    offset = C.c_uint64()
    call("nt_ipc_export", C.c_void_p(ptr), handle, C.byref(offset))
    return bytes(handle), int(offset.value)


def ipc_open(handle: bytes, offset: int) -> int:
    """Maps another process's exported buffer on the current device; returns its address."""
    buf = (C.c_ubyte * 64).from_buffer_copy(handle)
    out = C.c_void_p()
    call("nt_ipc_open", buf, C.c_uint64(offset), C.byref(out))
    return int(out.value)


def ipc_close(ptr: int) -> None:
    call("nt_ipc_close", C.c_void_p(ptr))


def peer_copy(src: list[int], dst: list[int], bytes_each: int, stream=None) -> None:
    """src[k] -> dst[k] for every k, ``bytes_each`` bytes each, by SM loads/stores (32-byte when every pointer and the size allow, else 16-byte)."""
    n = len(src)
    call("nt_peer_copy", (C.c_void_p * n)(*src), (C.c_void_p * n)(*dst), n, int(bytes_each), stream_handle(stream))


def can_access_peer(peer: int) -> bool:
    ok = C.c_int32()
    call("nt_can_access_peer", int(peer), C.byref(ok))
    return bool(ok.value)
