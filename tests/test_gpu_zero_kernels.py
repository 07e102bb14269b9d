"""Single-GPU parity of the two ZeRO-1 peer-memory kernels.

The kernels only see pointers, so local buffers stand in for the other ranks' memory:
``nt_zero_reduce_scatter_stats`` gets R separate local gradient buffers as its R sources,
``nt_adamw_mt_push`` gets local buffers as its peer copies. The multi-GPU choreography
(IPC mappings, barriers) is covered by test_gpu_zero.py.
"""
import numpy as np
import pytest
import torch

from namitorch_b200 import _native as N
from namitorch_b200.flat import CHUNK, segment_table, stats_tensor, upload
from namitorch_b200.optim._engine import CorrectionTable
from namitorch_b200.zero import CudaShardKernels
from oracle.casts import round_to_bf16

pytestmark = pytest.mark.gpu

DTYPES = {torch.bfloat16: "bf16", torch.float16: "f16", torch.float32: "f32"}


def _round(x: np.ndarray, dtype) -> np.ndarray:
    """float32 -> dtype (round to nearest even) -> float32."""
    if dtype == torch.bfloat16:
        return round_to_bf16(x)
    if dtype == torch.float16:
        return x.astype(np.float16).astype(np.float32)
    return x.astype(np.float32)


def _expected(sources: list[np.ndarray], dtype, average: bool, scale):
    total = sources[0].astype(np.float32)
    for src in sources[1:]:
        total = total + src.astype(np.float32)
    if average:
        n = len(sources)
        total = total * np.float32(1.0 / n) if n & (n - 1) == 0 else total / np.float32(n)
    dest = _round(total, dtype)
    u = dest if scale is None else dest / np.float32(scale)
    finite = np.isfinite(u)
    stats = {"sumsq": float(np.sum(np.square(u[finite].astype(np.float64)))),
             "nonfinite": float(np.count_nonzero(~finite)), "nan": float(np.count_nonzero(np.isnan(u))),
             "maxabs": float(np.max(np.abs(u[~np.isnan(u)]), initial=0.0))}
    return dest, stats


def _run_reduce(ranks, dtype, count, *, average=True, scale=None, poison=False, seed=0, offset_bytes=0):
    rng = np.random.default_rng(seed)
    host = []
    for q in range(ranks):
        g = rng.normal(0.0, 1.0, count).astype(np.float32) * np.float32(scale or 1.0) * np.float32(0.25)
        if poison and q == ranks - 1:
            g[count // 3] = np.inf
            g[count // 2] = np.nan
        host.append(_round(g, dtype))
    # offset_bytes shifts every source and the destination off the allocation's start: 16
    # leaves them 16- but not 32-byte aligned, so the kernel takes its 16-byte accesses.
    pad = offset_bytes // torch.empty(0, dtype=dtype).element_size()
    dev = []
    for h in host:
        t = torch.empty(count + pad, dtype=dtype, device="cuda")
        t[pad:] = torch.from_numpy(h).to("cuda").to(dtype)
        dev.append(t[pad:])
    dest = torch.full((count + pad,), 7.0, dtype=dtype, device="cuda")[pad:]
    stats = stats_tensor(torch.device("cuda"))
    scale_t = None if scale is None else torch.tensor([scale], dtype=torch.float32, device="cuda")
    k = CudaShardKernels(torch.device("cuda"))
    k.reduce_stats([t.data_ptr() for t in dev], dest, stats, scale=scale_t, average=average)
    torch.cuda.synchronize()
    got = dest.float().cpu().numpy()
    want, want_stats = _expected(host, dtype, average, scale)
    return got, want, stats.cpu().numpy(), want_stats


@pytest.mark.parametrize("dtype", list(DTYPES), ids=list(DTYPES.values()))
@pytest.mark.parametrize("ranks", [1, 2, 3, 4, 5, 8])
def test_reduce_scatter_stats_matches_rank_order_f32_sum(cuda_device, ranks, dtype):
    # 1,000,003 elements: not a multiple of the vector width, so the scalar tail runs too.
    got, want, stats, ref = _run_reduce(ranks, dtype, 1_000_003, scale=1024.0, seed=ranks)
    np.testing.assert_array_equal(got, want)
    s = dict(zip(N.STATS_FIELDS, stats))
    assert s["nonfinite"] == ref["nonfinite"] == 0 and s["nan"] == ref["nan"] == 0
    assert s["maxabs"] == ref["maxabs"]
    assert abs(s["sumsq"] - ref["sumsq"]) <= 1e-12 * ref["sumsq"]


@pytest.mark.parametrize("dtype", list(DTYPES), ids=list(DTYPES.values()))
@pytest.mark.parametrize("ranks", [2, 4, 8])
def test_reduce_scatter_stats_16_byte_aligned_sources(cuda_device, ranks, dtype):
    """Sources and destination 16 bytes past a 32-byte boundary: the 16-byte access path,
    with the same results as the 32-byte one."""
    got, want, stats, ref = _run_reduce(ranks, dtype, 500_009, scale=1024.0, seed=10 + ranks, offset_bytes=16)
    np.testing.assert_array_equal(got, want)
    s = dict(zip(N.STATS_FIELDS, stats))
    assert s["maxabs"] == ref["maxabs"] and abs(s["sumsq"] - ref["sumsq"]) <= 1e-12 * ref["sumsq"]


@pytest.mark.parametrize("average,scale", [(False, None), (True, 3.0), (False, 65536.0)])
def test_reduce_scatter_stats_scale_kinds_and_nonfinite(cuda_device, average, scale):
    got, want, stats, ref = _run_reduce(4, torch.bfloat16, 262_147, average=average, scale=scale, poison=True)
    np.testing.assert_array_equal(got, want)   # NaN positions compare equal
    s = dict(zip(N.STATS_FIELDS, stats))
    assert s["nonfinite"] == ref["nonfinite"] == 2 and s["nan"] == ref["nan"] == 1
    assert s["maxabs"] == ref["maxabs"]
    assert abs(s["sumsq"] - ref["sumsq"]) <= 1e-12 * ref["sumsq"]


def test_reduce_scatter_stats_empty_shard(cuda_device):
    k = CudaShardKernels(torch.device("cuda"))
    src = torch.zeros(8, dtype=torch.bfloat16, device="cuda")
    dest = torch.zeros(0, dtype=torch.bfloat16, device="cuda")
    stats = stats_tensor(torch.device("cuda"))
    k.reduce_stats([src.data_ptr(), src.data_ptr()], dest, stats, scale=None, average=True)
    torch.cuda.synchronize()
    s = dict(zip(N.STATS_FIELDS, stats.cpu().numpy()))
    assert s["sumsq"] == 0 and s["nonfinite"] == 0 and s["maxabs"] == 0


def test_reduce_scatter_rejects_misaligned_and_bad_rank_counts(cuda_device):
    k = CudaShardKernels(torch.device("cuda"))
    buf = torch.zeros(64, dtype=torch.bfloat16, device="cuda")
    dest = torch.zeros(32, dtype=torch.bfloat16, device="cuda")
    stats = stats_tensor(torch.device("cuda"))
    with pytest.raises(ValueError, match="16-byte aligned"):
        k.reduce_stats([buf.data_ptr(), buf.data_ptr() + 2], dest, stats, scale=None, average=True)
    with pytest.raises(ValueError, match="num_ranks"):
        k.reduce_stats([buf.data_ptr()] * 9, dest, stats, scale=None, average=True)


def _update(push_to, grads, p0, total, seg_rows, *, scale=None, stats=None, max_norm=None):
    device = torch.device("cuda")
    k = CudaShardKernels(device)
    corr = CorrectionTable(device)
    row = corr.row(0.9, 0.999)
    corr.ensure(2)
    group = N.AdamWGroup(lr=np.float32(1e-3), beta1=np.float32(0.9), beta2=np.float32(0.999),
                         one_minus_beta1=np.float32(0.1), one_minus_beta2=np.float32(1 - 0.999),
                         eps=np.float32(1e-8), weight_decay=np.float32(0.1),
                         decay_factor=np.float32(1 - 1e-3 * 0.1), maximize=0, decay_mode=N.NT_DECAY_DECOUPLED,
                         update_parameter=1, correction_row=row)
    master = torch.from_numpy(p0.copy()).to(device)
    m = torch.zeros(total, dtype=torch.float32, device=device)
    v = torch.zeros(total, dtype=torch.float32, device=device)
    copy = torch.zeros(total, dtype=torch.bfloat16, device=device)
    steps = torch.zeros(len(seg_rows), dtype=torch.int32, device=device)
    rows = [(grads.data_ptr() + off * 2, off, n, 0, slot) for slot, (off, n) in enumerate(seg_rows)]
    table, nchunks = segment_table(rows, CHUNK)
    segs = upload(table, device)
    peers = [torch.zeros(total, dtype=torch.bfloat16, device=device) for _ in range(push_to)]
    k.update(master=master, exp_avg=m, exp_avg_sq=v, copy=copy, grad_dtype=torch.bfloat16, segments=segs,
             num_segments=len(rows), num_chunks=nchunks, steps=steps, corrections=corr.tensor,
             capacity=corr.capacity, scale=scale, stats=stats, skip=stats is not None,
             max_norm=max_norm, groups=[group], peers=[p.data_ptr() for p in peers] or None)
    torch.cuda.synchronize()
    return master, m, v, copy, steps, peers


@pytest.mark.parametrize("npeers", [1, 3, 7])
def test_adamw_push_writes_every_copy_and_matches_plain_update(cuda_device, npeers):
    rng = np.random.default_rng(npeers)
    total = 3 * CHUNK + 1000
    # Segments: vector-aligned, ragged (odd count: the scalar tail), and a late start.
    seg_rows = [(0, 2 * CHUNK + 5), (2 * CHUNK + 64, 777), (2 * CHUNK + 1024, total - 2 * CHUNK - 1024)]
    p0 = rng.normal(0, 0.02, total).astype(np.float32)
    g = torch.from_numpy(rng.normal(0, 1e-3, total).astype(np.float32) * np.float32(1024)).to("cuda")
    g = g.to(torch.bfloat16)
    scale = torch.tensor([1024.0], dtype=torch.float32, device="cuda")
    stats = stats_tensor(torch.device("cuda"))
    stats[N.STATS_FIELDS.index("norm")] = 2.5   # clip coefficient 0.4
    base = _update(0, g, p0, total, seg_rows, scale=scale, stats=stats, max_norm=1.0)
    pushed = _update(npeers, g, p0, total, seg_rows, scale=scale, stats=stats, max_norm=1.0)
    for a, b in zip(base[:5], pushed[:5]):   # master, m, v, copy, steps: bit-identical
        assert torch.equal(a.view(torch.uint8), b.view(torch.uint8))
    covered = torch.zeros(total, dtype=torch.bool, device="cuda")
    for off, n in seg_rows:
        covered[off:off + n] = True
    for peer in pushed[5]:
        assert torch.equal(peer[covered], pushed[3][covered])     # every updated element arrived
        assert not torch.any(peer[~covered].float() != 0)         # nothing outside the segments
    # The pushed copy is the bf16 rounding of the updated master.
    assert torch.equal(pushed[3][covered], pushed[0][covered].to(torch.bfloat16))


def test_adamw_push_skips_with_found_inf(cuda_device):
    total = CHUNK
    p0 = np.full(total, 0.5, np.float32)
    g = torch.ones(total, dtype=torch.bfloat16, device="cuda")
    stats = stats_tensor(torch.device("cuda"))
    stats[N.STATS_FIELDS.index("found_inf")] = 1.0
    master, m, v, copy, steps, peers = _update(2, g, p0, total, [(0, total)], stats=stats)
    assert torch.equal(master.cpu(), torch.from_numpy(p0))
    assert int(steps[0]) == 0
    for peer in peers:
        assert not torch.any(peer.float() != 0)


@pytest.mark.parametrize("count,bytes_each,offset", [(1, 1 << 20, 0), (2, (1 << 20) + 64, 0), (3, (1 << 20) + 48, 0), (2, 4096 + 32, 16),
                                                     (4, 16, 0)])
def test_peer_copy_copies_every_range(cuda_device, count, bytes_each, offset):
    """nt_peer_copy on local buffers: 32-byte accesses (aligned pointers, size a multiple of
    32) and 16-byte ones (pointers 16 bytes past a 32-byte boundary, or an odd 16-byte
    count) copy every byte of every range and nothing past it."""
    src = [torch.randint(0, 256, (bytes_each + offset + 64,), dtype=torch.uint8, device="cuda") for _ in range(count)]
    dst = [torch.zeros(bytes_each + offset + 64, dtype=torch.uint8, device="cuda") for _ in range(count)]
    N.peer_copy([s.data_ptr() + offset for s in src], [d.data_ptr() + offset for d in dst], bytes_each)
    torch.cuda.synchronize()
    for s, d in zip(src, dst):
        assert torch.equal(d[offset:offset + bytes_each], s[offset:offset + bytes_each])
        assert not torch.any(d[:offset]) and not torch.any(d[offset + bytes_each:])


def test_peer_copy_rejects_bad_arguments(cuda_device):
    buf = torch.zeros(256, dtype=torch.uint8, device="cuda")
    with pytest.raises(ValueError, match="multiple of 16"):
        N.peer_copy([buf.data_ptr()], [buf.data_ptr() + 128], 24)
    with pytest.raises(ValueError, match="16-byte aligned"):
        N.peer_copy([buf.data_ptr() + 8], [buf.data_ptr() + 128], 32)
    with pytest.raises(ValueError, match="count"):
        N.peer_copy([], [], 32)
