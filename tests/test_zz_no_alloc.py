"""Allocation-free gradient statistics, checked against the allocating entry point.

Some callers of this library cannot allocate device memory themselves. Examples: a host
whose device memory all belongs to its own pool, a plugin that runs inside another
runtime's allocator, or a C/FFI caller without the CUDA allocation calls. For them,
``nt_grad_stats_noalloc`` keeps its scratch (block partials, last-block ticket, span
table) in a static device array inside the library, so the caller only passes the
gradients and the output record.

This test calls it through the C ABI twice in a row, with different data each time.
The array keeps the previous call's contents, so the second call shows that nothing
stale leaks through. Each result is compared with ``nt_grad_stats`` (caller-allocated
workspace) on the same inputs, to the 1e-12 relative bound the other norm tests use.
The file is named to be collected last, so a failure here comes after every other test
has already run.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from namitorch_b200 import _native as N
from namitorch_b200.flat import CHUNK, span_table, upload

pytestmark = pytest.mark.gpu
FIELDS = ["sumsq", "nonfinite", "nan", "maxabs", "norm", "found_inf"]


def _grads(seed, inject_inf):
    rng = np.random.default_rng(seed)
    out = []
    for n in (5, 8, 1000, 8191, 8193, 0, 300001):
        g = rng.normal(0, 1e-2, n).astype(np.float32) * 1024.0
        if inject_inf and n == 1000:
            g[17] = np.inf
        out.append(torch.from_numpy(g).cuda().to(torch.bfloat16))
    return out


def _allocating(grads, scale, p):
    pairs = [(g.data_ptr(), g.numel()) for g in grads if g.numel()]
    table, nchunks = span_table(pairs, CHUNK)
    spans = upload(table, torch.device("cuda", 0))
    stats = torch.zeros(N.STATS_DOUBLES, dtype=torch.float64, device="cuda")
    ws_bytes = int(N.load().nt_grad_stats_workspace_size())
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    passes = [0] if p in (2.0, float("inf")) else [0, 1]
    for k in passes:
        args = N.GradStatsArgs(spans=spans.data_ptr(), num_spans=len(pairs), chunk_elems=CHUNK, num_chunks=nchunks,
                               dtype=N.NT_BF16, scale=scale.data_ptr(), pass_=k, norm_type=p,
                               finalize=int(k == passes[-1]), stats=stats.data_ptr(), workspace=ws.data_ptr(),
                               workspace_bytes=ws_bytes)
        N.check(N.load().nt_grad_stats(ctypes.byref(args), N.stream_handle()))
    return stats


def _noalloc(grads, scale, p):
    lib = N.load()
    host = (N.Span * len(grads))(*[N.Span(ptr=g.data_ptr() if g.numel() else None, count=g.numel(), chunk_begin=0)
                                   for g in grads])
    stats = torch.zeros(N.STATS_DOUBLES, dtype=torch.float64, device="cuda")
    N.check(lib.nt_grad_stats_noalloc(host, len(grads), N.NT_BF16, ctypes.c_void_p(scale.data_ptr()), p,
                                      ctypes.c_void_p(stats.data_ptr()), ctypes.c_void_p(N.stream_handle())))
    return stats


def _close(a, b):
    if math.isnan(a) or math.isnan(b):
        return math.isnan(a) and math.isnan(b)
    if math.isinf(a) or math.isinf(b):
        return a == b
    return abs(a - b) <= 1e-12 * max(abs(a), abs(b))


@pytest.mark.parametrize("p", [2.0, 3.0])
def test_noalloc_stats_match_allocating_entry_point_on_two_calls(p):
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    torch.cuda.set_device(0)
    scale = torch.tensor([1024.0], device="cuda")
    assert N.load().nt_grad_stats_noalloc_scratch_bytes() < 64 * 1024
    for call, inject in enumerate((False, True)):
        grads = _grads(seed=call + 10 * int(p), inject_inf=inject)
        ours = _noalloc(grads, scale, p).cpu().numpy()
        ref = _allocating(grads, scale, p).cpu().numpy()
        for name in FIELDS:
            i = N.STATS_FIELDS.index(name)
            assert _close(float(ours[i]), float(ref[i])), (call, name, ours[i], ref[i])
        assert ours[N.STATS_FIELDS.index("found_inf")] == (1.0 if inject else 0.0)


def test_noalloc_rejects_more_spans_than_its_table_holds():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    lib = N.load()
    n = 65
    g = torch.zeros(8, dtype=torch.bfloat16, device="cuda")
    host = (N.Span * n)(*[N.Span(ptr=g.data_ptr(), count=8, chunk_begin=0) for _ in range(n)])
    stats = torch.zeros(N.STATS_DOUBLES, dtype=torch.float64, device="cuda")
    rc = lib.nt_grad_stats_noalloc(host, n, N.NT_BF16, None, 2.0, ctypes.c_void_p(stats.data_ptr()), None)
    assert rc == N.NT_EINVAL
    assert "exceed the maximum of 64" in N.last_error()
