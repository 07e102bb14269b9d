"""Flat-buffer layout and device work tables.

Parameters are packed into flat arenas (fp32 master, exp_avg, exp_avg_sq and an optional
bf16/fp16 model copy) with every tensor starting on a 64-element boundary (256 bytes of
fp32), so each one is a 16-byte aligned run the kernels read with 128-bit loads. The
Python-side tensors become views into the arenas: nothing is flattened or copied per step.

Work tables tell the multi-tensor kernels where each segment / span lives; they are
uploaded once and reused for as long as the gradient pointers stay the same.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as N
from .errors import NamiTorchCUDAOutOfMemoryError

def zeroed_arena(numel: int, dtype: torch.dtype, device) -> torch.Tensor:
    """A zero-filled flat device buffer. An allocation failure raises the reference's
    NamiTorchCUDAOutOfMemoryError (namitorch/backends/_cuda_memory.py:8-21) with the requested
    bytes, the bytes the allocator holds (allocated / reserved) and the device's free / total
    bytes, in place of torch's own out-of-memory error."""
    try:
        return torch.zeros(int(numel), dtype=dtype, device=device)
    except torch.OutOfMemoryError as error:
        raise out_of_memory(torch.device(device), int(numel) * torch.empty((), dtype=dtype).element_size()) from error


def out_of_memory(device: torch.device, requested: int) -> NamiTorchCUDAOutOfMemoryError:
    """The reference's out-of-memory error for a failed request of `requested` bytes."""
    allocated = reserved = free = total = None
    try:
        allocated = int(torch.cuda.memory_allocated(device))
        reserved = int(torch.cuda.memory_reserved(device))
        free, total = (int(x) for x in torch.cuda.mem_get_info(device))
    except Exception:   # the error still carries what could be read
        pass
    return NamiTorchCUDAOutOfMemoryError(str(device), requested, allocated, reserved, free, total)


ALIGN = 64          # elements: every segment starts on a 256-byte boundary of an fp32 arena
CHUNK = 8192        # elements per work chunk of the multi-tensor kernels

SEGMENT_DTYPE = np.dtype([("grad", "<u8"), ("offset", "<i8"), ("count", "<i8"), ("chunk_begin", "<i8"),
                          ("group", "<i4"), ("step_slot", "<i4")])
SPAN_DTYPE = np.dtype([("ptr", "<u8"), ("count", "<i8"), ("chunk_begin", "<i8")])
assert SEGMENT_DTYPE.itemsize == 40 and SPAN_DTYPE.itemsize == 24


def round_up(value: int, multiple: int) -> int:
    return (value + multiple - 1) // multiple * multiple


def chunks_of(count: int, chunk: int = CHUNK) -> int:
    return (count + chunk - 1) // chunk


@dataclass
class FlatLayout:
    """Element offsets of a list of tensors packed with ALIGN-element alignment."""
    numels: list[int]
    offsets: list[int]
    total: int

    @classmethod
    def build(cls, numels: list[int], align: int = ALIGN, pad_to: int = ALIGN) -> "FlatLayout":
        offsets = []
        cursor = 0
        for n in numels:
            offsets.append(cursor)
            cursor = round_up(cursor + int(n), align)
        return cls(list(map(int, numels)), offsets, round_up(max(cursor, 1), pad_to))


def segment_table(entries: list[tuple[int, int, int, int, int]], chunk: int = CHUNK) -> tuple[np.ndarray, int]:
    """entries: (grad_ptr, arena_offset, count, group, step_slot) -> (table, total chunks)."""
    table = np.zeros(len(entries), SEGMENT_DTYPE)
    begin = 0
    for i, (ptr, offset, count, group, slot) in enumerate(entries):
        table[i] = (ptr, offset, count, begin, group, slot)
        begin += chunks_of(count, chunk)
    return table, begin


def span_table(spans: list[tuple[int, int]], chunk: int = CHUNK) -> tuple[np.ndarray, int]:
    """spans: (ptr, count) -> (table, total chunks)."""
    table = np.zeros(len(spans), SPAN_DTYPE)
    begin = 0
    for i, (ptr, count) in enumerate(spans):
        table[i] = (ptr, count, begin)
        begin += chunks_of(count, chunk)
    return table, begin


def upload(table: np.ndarray, device: torch.device) -> torch.Tensor:
    host = torch.from_numpy(np.ascontiguousarray(table).view(np.uint8).copy())
    return host.to(device, non_blocking=False)


def stats_tensor(device: torch.device) -> torch.Tensor:
    """A fresh device nt_stats record (8 float64)."""
    return torch.zeros(N.STATS_DOUBLES, dtype=torch.float64, device=device)


def stats_field(stats: torch.Tensor, name: str) -> torch.Tensor:
    i = N.STATS_FIELDS.index(name)
    return stats[i]


class WorkspaceCache:
    """Zero-initialised kernel workspaces, one per (device, stream, kind).

    A workspace is only ever used by launches on its own stream, which the stream
    serialises, so one buffer per stream is enough."""

    def __init__(self):
        self._buffers: dict[tuple, torch.Tensor] = {}
        self._lock = threading.Lock()

    def get(self, kind: str, nbytes: int, device: torch.device, stream=None) -> torch.Tensor:
        stream = torch.cuda.current_stream(device) if stream is None else stream
        key = (kind, device.index, int(stream.cuda_stream))
        with self._lock:
            buf = self._buffers.get(key)
            if buf is None or buf.numel() < nbytes:
                buf = torch.zeros(round_up(nbytes, 256), dtype=torch.uint8, device=device)
                self._buffers[key] = buf
            return buf


WORKSPACES = WorkspaceCache()


def stats_workspace(device: torch.device) -> torch.Tensor:
    return WORKSPACES.get("stats", int(N.load().nt_grad_stats_workspace_size()), device)


def xent_workspace(device: torch.device) -> torch.Tensor:
    return WORKSPACES.get("xent", int(N.load().nt_xent_workspace_size()), device)


def launch_grad_stats(spans_dev: torch.Tensor, num_spans: int, num_chunks: int, dtype: torch.dtype,
                      stats: torch.Tensor, *, scale: torch.Tensor | None = None, norm_type: float = 2.0,
                      finalize: bool = True) -> torch.Tensor:
    """Runs the statistics reduction (one pass, two for a general p) into ``stats``."""
    device = stats.device
    ws = stats_workspace(device)
    stream = N.stream_handle()
    passes = [0] if (norm_type == 2.0 or norm_type == float("inf")) else [0, 1]
    for p in passes:
        args = N.GradStatsArgs(
            spans=spans_dev.data_ptr() if num_spans else None, num_spans=num_spans, chunk_elems=CHUNK,
            num_chunks=num_chunks, dtype=N.dtype_code(dtype), scale=None if scale is None else scale.data_ptr(),
            pass_=p, norm_type=float(norm_type), finalize=int(finalize and p == passes[-1]),
            stats=stats.data_ptr(), workspace=ws.data_ptr(), workspace_bytes=ws.numel())
        N.call("nt_grad_stats", N.C.byref(args), stream)
    return stats


# ---- gradient-list helpers (statistics and in-place transforms over arbitrary tensors) ------
_SPAN_CACHE: dict[tuple, tuple[torch.Tensor, int, int]] = {}


def _spans_for(grads: list[torch.Tensor]) -> tuple[torch.Tensor | None, int, int]:
    device = grads[0].device if grads else None
    key = (device, tuple((g.data_ptr(), g.numel()) for g in grads))
    hit = _SPAN_CACHE.get(key)
    if hit is not None:
        return hit
    pairs = [(g.data_ptr(), g.numel()) for g in grads if g.numel()]
    if not pairs:
        result = (None, 0, 0)
    else:
        table, nchunks = span_table(pairs, CHUNK)
        result = (upload(table, device), len(pairs), nchunks)
    if len(_SPAN_CACHE) > 64:
        _SPAN_CACHE.clear()
    _SPAN_CACHE[key] = result
    return result


def _by_dtype(grads: list[torch.Tensor]) -> dict[torch.dtype, list[torch.Tensor]]:
    out: dict[torch.dtype, list[torch.Tensor]] = {}
    for g in grads:
        out.setdefault(g.dtype, []).append(g if g.is_contiguous() else g.contiguous())
    return out


def grad_stats_for(grads: list[torch.Tensor], *, scale: torch.Tensor | None = None, norm_type: float = 2.0,
                   device: torch.device | None = None) -> torch.Tensor:
    """found_inf / max|g| / total norm of the (unscaled) gradients, as a new device record."""
    if device is None:
        device = grads[0].device if grads else (scale.device if scale is not None else
                                                torch.device("cuda", torch.cuda.current_device()))
    groups = _by_dtype(grads)
    stats = stats_tensor(device)
    with torch.cuda.device(device):
        if len(groups) <= 1:
            dtype, members = next(iter(groups.items())) if groups else (torch.float32, [])
            spans, n, chunks = _spans_for(members)
            return launch_grad_stats(spans, n, chunks, dtype, stats, scale=scale, norm_type=norm_type, finalize=True)
        # Several dtypes: reduce each, combine on the device, then finalize once.
        parts = []
        for dtype, members in groups.items():
            spans, n, chunks = _spans_for(members)
            part = stats_tensor(device)
            launch_grad_stats(spans, n, chunks, dtype, part, scale=scale, norm_type=2.0, finalize=False)
            parts.append((dtype, members, part))
        stacked = torch.stack([p for _, _, p in parts])
        idx = {name: N.STATS_FIELDS.index(name) for name in N.STATS_FIELDS}
        for name in ("sumsq", "nonfinite", "nan"):
            stats[idx[name]] = stacked[:, idx[name]].sum()
        stats[idx["maxabs"]] = stacked[:, idx["maxabs"]].max()
        if not (norm_type == 2.0 or norm_type == float("inf")):
            for dtype, members, part in parts:
                part[idx["maxabs"]] = stats[idx["maxabs"]]
                spans, n, chunks = _spans_for(members)
                ws = stats_workspace(device)
                args = N.GradStatsArgs(spans=spans.data_ptr() if n else None, num_spans=n, chunk_elems=CHUNK,
                                       num_chunks=chunks, dtype=N.dtype_code(dtype),
                                       scale=None if scale is None else scale.data_ptr(), pass_=1,
                                       norm_type=float(norm_type), finalize=0, stats=part.data_ptr(),
                                       workspace=ws.data_ptr(), workspace_bytes=ws.numel())
                N.call("nt_grad_stats", N.C.byref(args), N.stream_handle())
            stats[idx["powsum"]] = torch.stack([p[idx["powsum"]] for _, _, p in parts]).sum()
        N.call("nt_grad_stats_finalize", stats.data_ptr(), float(norm_type), N.stream_handle())
    return stats


def launch_transform(grads: list[torch.Tensor], *, scale: torch.Tensor | None = None,
                     stats: torch.Tensor | None = None, max_norm: float | None = None,
                     clip_value: float | None = None) -> None:
    """In-place unscale / clip-by-norm (or clip-by-value) of every gradient."""
    if not grads:
        return
    device = grads[0].device
    with torch.cuda.device(device):
        by_dtype: dict[torch.dtype, list[tuple[torch.Tensor, torch.Tensor]]] = {}
        for g in grads:
            work = g if g.is_contiguous() else g.contiguous()
            by_dtype.setdefault(g.dtype, []).append((g, work))
        for dtype, pairs in by_dtype.items():
            spans, n, chunks = _spans_for([w for _, w in pairs])
            if n == 0:
                continue
            if clip_value is not None:
                N.call("nt_grad_clip_value", spans.data_ptr(), n, CHUNK, chunks, N.dtype_code(dtype),
                       float(clip_value), N.stream_handle())
            else:
                N.call("nt_grad_transform", spans.data_ptr(), n, CHUNK, chunks, N.dtype_code(dtype),
                       None if scale is None else scale.data_ptr(), None if stats is None else stats.data_ptr(),
                       int(max_norm is not None), float(max_norm or 0.0), N.stream_handle())
            for g, w in pairs:
                if w is not g:
                    g.copy_(w)
