"""Allocation-free gradient statistics, checked against the allocating entry point.

Some callers of this library cannot allocate device memory themselves. Examples: a host
whose device memory all belongs to its own pool, a plugin that runs inside another
runtime's allocator, or a C/FFI caller without the CUDA allocation calls. For them,
``nt_grad_stats_noalloc`` keeps its scratch (block partials, last-block ticket, span
table) in a static device array inside the library, so the caller only passes the
gradients and the output record.

These tests call it through the C ABI twice in a row, with different data each time.
The array keeps the previous call's contents, so the second call shows that nothing
stale leaks through. Each result is compared with ``nt_grad_stats`` (caller-allocated
workspace) on the same inputs, to the 1e-12 relative bound the other norm tests use,
for float32 / float16 / bfloat16 gradients, p = 2, 3 and inf, no spans at all, spans that
start off the 16-byte boundary and no loss scale. The array's device address belongs to
a CUDA context, so one test also runs the entry point in contexts created with the
driver API (a child process that uses no torch). The file is named to be collected last,
so a failure here comes after every other test has already run.
"""
import ctypes
import math
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest
import torch

from namitorch_b200 import _native as N
from namitorch_b200.flat import CHUNK, span_table, upload

pytestmark = pytest.mark.gpu
FIELDS = ["sumsq", "nonfinite", "nan", "maxabs", "norm", "found_inf"]
DTYPES = {"f32": (torch.float32, N.NT_F32), "f16": (torch.float16, N.NT_F16), "bf16": (torch.bfloat16, N.NT_BF16)}
REPO = Path(__file__).resolve().parents[1]


def _grads(seed, inject_inf, dtype, offset=0):
    """Seven gradients (one empty, several not a whole number of chunks); with ``offset``,
    each starts ``offset`` elements into its own buffer, off the 16-byte boundary."""
    rng = np.random.default_rng(seed)
    out = []
    for n in (5, 8, 1000, 8191, 8193, 0, 300001):
        g = rng.normal(0, 1e-2, n).astype(np.float32) * 1024.0
        if inject_inf and n == 1000:
            g[17] = np.inf
        full = torch.zeros(n + offset, dtype=dtype, device="cuda")
        full[offset:] = torch.from_numpy(g).cuda().to(dtype)
        out.append(full[offset:])
    return out


def _allocating(grads, scale, p, code):
    pairs = [(g.data_ptr(), g.numel()) for g in grads if g.numel()]
    table, nchunks = span_table(pairs, CHUNK)
    spans = upload(table, torch.device("cuda", 0))
    stats = torch.zeros(N.STATS_DOUBLES, dtype=torch.float64, device="cuda")
    ws_bytes = int(N.load().nt_grad_stats_workspace_size())
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device="cuda")
    passes = [0] if p in (2.0, float("inf")) else [0, 1]
    for k in passes:
        args = N.GradStatsArgs(spans=spans.data_ptr(), num_spans=len(pairs), chunk_elems=CHUNK, num_chunks=nchunks,
                               dtype=code, scale=None if scale is None else scale.data_ptr(), pass_=k, norm_type=p,
                               finalize=int(k == passes[-1]), stats=stats.data_ptr(), workspace=ws.data_ptr(),
                               workspace_bytes=ws_bytes)
        N.check(N.load().nt_grad_stats(ctypes.byref(args), N.stream_handle()))
    return stats


def _noalloc(grads, scale, p, code):
    lib = N.load()
    host = (N.Span * max(1, len(grads)))(*[N.Span(ptr=g.data_ptr() if g.numel() else None, count=g.numel(),
                                                  chunk_begin=0) for g in grads])
    stats = torch.full((N.STATS_DOUBLES,), 7.0, dtype=torch.float64, device="cuda")   # not zero on entry
    N.check(lib.nt_grad_stats_noalloc(host, len(grads), code,
                                      None if scale is None else ctypes.c_void_p(scale.data_ptr()), p,
                                      ctypes.c_void_p(stats.data_ptr()), ctypes.c_void_p(N.stream_handle())))
    return stats


def _close(a, b):
    if math.isnan(a) or math.isnan(b):
        return math.isnan(a) and math.isnan(b)
    if math.isinf(a) or math.isinf(b):
        return a == b
    return abs(a - b) <= 1e-12 * max(abs(a), abs(b))


def _compare(ours, ref, where):
    for name in FIELDS:
        i = N.STATS_FIELDS.index(name)
        assert _close(float(ours[i]), float(ref[i])), (where, name, ours[i], ref[i])


@pytest.fixture
def cuda0():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    torch.cuda.set_device(0)


@pytest.mark.parametrize("dtype", sorted(DTYPES))
@pytest.mark.parametrize("p", [2.0, 3.0, float("inf")])
def test_noalloc_stats_match_allocating_entry_point_on_two_calls(cuda0, p, dtype):
    torch_dtype, code = DTYPES[dtype]
    scale = torch.tensor([1024.0], device="cuda")
    assert N.load().nt_grad_stats_noalloc_scratch_bytes() < 64 * 1024
    for call, inject in enumerate((False, True)):
        grads = _grads(seed=call + 10 * int(min(p, 9)), inject_inf=inject, dtype=torch_dtype)
        ours = _noalloc(grads, scale, p, code).cpu().numpy()
        ref = _allocating(grads, scale, p, code).cpu().numpy()
        _compare(ours, ref, (dtype, p, call))
        assert ours[N.STATS_FIELDS.index("found_inf")] == (1.0 if inject else 0.0)


@pytest.mark.parametrize("p", [2.0, 3.0])
def test_noalloc_unaligned_spans_and_no_scale(cuda0, p):
    """Spans that start 3 elements into their buffers (the per-element edge path) and a
    NULL loss scale, twice in a row, against the allocating entry point."""
    for call in range(2):
        grads = _grads(seed=40 + call, inject_inf=bool(call), dtype=torch.bfloat16, offset=3)
        assert all(g.data_ptr() % 16 for g in grads if g.numel())
        ours = _noalloc(grads, None, p, N.NT_BF16).cpu().numpy()
        ref = _allocating(grads, None, p, N.NT_BF16).cpu().numpy()
        _compare(ours, ref, ("unaligned", p, call))


@pytest.mark.parametrize("p", [2.0, 3.0, float("inf")])
def test_noalloc_no_spans_gives_a_zero_norm(cuda0, p):
    """No gradients at all (and, before that, a call that leaves a non-zero record in the
    shared array): norm 0, nothing non-finite."""
    scale = torch.tensor([2.0], device="cuda")
    _noalloc(_grads(seed=5, inject_inf=True, dtype=torch.float32), scale, p, N.NT_F32)
    for grads in ([], [torch.zeros(0, dtype=torch.float32, device="cuda")]):
        ours = _noalloc(grads, scale, p, N.NT_F32).cpu().numpy()
        for name in ("sumsq", "nonfinite", "nan", "maxabs", "norm", "found_inf"):
            assert ours[N.STATS_FIELDS.index(name)] == 0.0, (len(grads), name, ours)


def test_noalloc_rejects_more_spans_than_its_table_holds(cuda0):
    lib = N.load()
    n = 65
    g = torch.zeros(8, dtype=torch.bfloat16, device="cuda")
    host = (N.Span * n)(*[N.Span(ptr=g.data_ptr(), count=8, chunk_begin=0) for _ in range(n)])
    stats = torch.zeros(N.STATS_DOUBLES, dtype=torch.float64, device="cuda")
    rc = lib.nt_grad_stats_noalloc(host, n, N.NT_BF16, None, 2.0, ctypes.c_void_p(stats.data_ptr()), None)
    assert rc == N.NT_EINVAL
    assert "exceed the maximum of 64" in N.last_error()


# A child process that uses the driver API only: it runs the entry point in the primary
# context, in two contexts it creates (the second may reuse the first one's handle value)
# and in the primary context again. Each run must give the same record, and the sum of
# squares must match NumPy's.
_CONTEXT_SCRIPT = textwrap.dedent(r"""
    import ctypes as C, sys
    import numpy as np
    sys.path.insert(0, sys.argv[1])
    from namitorch_b200 import _native as N

    cu = C.CDLL("libcuda.so.1")
    def ok(rc, what):
        if rc != 0:
            raise SystemExit(f"{what} failed with CUresult {rc}")
    ok(cu.cuInit(0), "cuInit")
    dev = C.c_int()
    ok(cu.cuDeviceGet(C.byref(dev), 0), "cuDeviceGet")
    lib = N.load()
    rng = np.random.default_rng(3)
    host = [rng.normal(0, 1, n).astype(np.float32) for n in (7, 8192, 100003)]
    want = sum(float(np.sum(h.astype(np.float64) ** 2)) for h in host)

    def run():
        ptrs = []
        for h in host:
            p = C.c_uint64()
            ok(cu.cuMemAlloc_v2(C.byref(p), C.c_size_t(h.nbytes)), "cuMemAlloc")
            ok(cu.cuMemcpyHtoD_v2(p, h.ctypes.data_as(C.c_void_p), C.c_size_t(h.nbytes)), "cuMemcpyHtoD")
            ptrs.append(p)
        out = C.c_uint64()
        ok(cu.cuMemAlloc_v2(C.byref(out), C.c_size_t(8 * N.STATS_DOUBLES)), "cuMemAlloc")
        spans = (N.Span * len(host))(*[N.Span(ptr=p.value, count=h.size, chunk_begin=0) for p, h in zip(ptrs, host)])
        rc = lib.nt_grad_stats_noalloc(spans, len(host), N.NT_F32, None, 2.0, C.c_void_p(out.value), None)
        if rc != 0:
            raise SystemExit(f"nt_grad_stats_noalloc: {rc} {N.last_error()}")
        ok(cu.cuCtxSynchronize(), "cuCtxSynchronize")
        rec = np.zeros(N.STATS_DOUBLES, np.float64)
        ok(cu.cuMemcpyDtoH_v2(rec.ctypes.data_as(C.c_void_p), out, C.c_size_t(rec.nbytes)), "cuMemcpyDtoH")
        for p in ptrs + [out]:
            ok(cu.cuMemFree_v2(p), "cuMemFree")
        return rec

    primary = C.c_void_p()
    ok(cu.cuDevicePrimaryCtxRetain(C.byref(primary), dev), "cuDevicePrimaryCtxRetain")
    ok(cu.cuCtxSetCurrent(primary), "cuCtxSetCurrent")
    records = [run()]
    for _ in range(2):
        ctx = C.c_void_p()
        ok(cu.cuCtxCreate_v2(C.byref(ctx), 0, dev), "cuCtxCreate")
        records.append(run())
        ok(cu.cuCtxDestroy_v2(ctx), "cuCtxDestroy")
    ok(cu.cuCtxSetCurrent(primary), "cuCtxSetCurrent")
    records.append(run())
    ok(cu.cuDevicePrimaryCtxRelease_v2(dev), "cuDevicePrimaryCtxRelease")
    sumsq = N.STATS_FIELDS.index("sumsq")
    for rec in records[1:]:
        assert np.array_equal(rec, records[0]), (rec, records[0])
    assert abs(records[0][sumsq] - want) <= 1e-10 * want, (records[0][sumsq], want)
    assert records[0][N.STATS_FIELDS.index("found_inf")] == 0.0
    print("contexts ok", len(records))
""")


def test_noalloc_scratch_address_follows_the_current_context(cuda0):
    result = subprocess.run([sys.executable, "-c", _CONTEXT_SCRIPT, str(REPO)], capture_output=True, text=True,
                            timeout=300)
    assert result.returncode == 0, result.stdout + result.stderr
    assert "contexts ok 4" in result.stdout
