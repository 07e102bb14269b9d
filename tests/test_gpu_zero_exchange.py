"""The in-kernel cross-GPU exchanges of the ZeRO-1 step, on one GPU.

``nt_zero_reduce_scatter_exchange`` and ``nt_adamw_mt_push_exchange`` wait on flags that
other ranks write into this rank's mailbox. One kernel runs per test and nothing runs
beside it: the other ranks' side is written into the mailbox by the host beforehand (a rank
that has already signalled), or never (a rank that stopped), and local buffers stand in for
their memory. Checked: the reduce-scatter with its statistics exchange gives the record of
``nt_zero_reduce_scatter_stats`` + finalize for one rank and the rank-order sum of every
rank's totals for two; each kernel signals its own flags (and statistics) into every
mailbox; a wait that nothing satisfies ends after the bound with the error word set and
the step skipped, and the device stays usable. The multi-GPU runs are test_gpu_zero.py and
the bench's self-check at N > 1.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

from namitorch_b200 import _native as N
from namitorch_b200.flat import CHUNK, segment_table, stats_tensor, upload
from namitorch_b200.optim._engine import CorrectionTable
from namitorch_b200.zero import CudaShardKernels

pytestmark = pytest.mark.gpu
MAILBOX_BYTES = ctypes.sizeof(N.ZeroMailbox)
FLAG_SLOTS = 3 * N.NT_MAX_RANKS          # int64 slots before the statistics


def _mailbox():
    return torch.zeros(MAILBOX_BYTES, dtype=torch.uint8, device="cuda")


def _flag(box, kind, rank):
    return int(box.view(torch.int64)[kind * N.NT_MAX_RANKS + rank].item())


def _set_flag(box, kind, rank, epoch):
    box.view(torch.int64)[kind * N.NT_MAX_RANKS + rank] = epoch


def _stats_slot(box, rank):
    return box.view(torch.float64)[FLAG_SLOTS + 4 * rank:FLAG_SLOTS + 4 * rank + 4]


def _sync(boxes, rank, epoch, error, timeout_ns=2_000_000_000):
    sync = N.ZeroSync(rank=rank, epoch=epoch, timeout_ns=timeout_ns, error=error.data_ptr())
    for q, box in enumerate(boxes):
        sync.mailboxes[q] = box.data_ptr()
    return sync


def _grads(ranks, count, seed):
    rng = np.random.default_rng(seed)
    return [torch.from_numpy(rng.normal(0, 1e-2, count).astype(np.float32) * np.float32(1024)).cuda()
            .to(torch.bfloat16) for _ in range(ranks)]


def test_exchange_for_one_rank_matches_the_plain_reduce_and_finalize(cuda_device):
    k = CudaShardKernels(cuda_device)
    src = _grads(1, 300_001, 1)
    scale = torch.tensor([1024.0], device="cuda")
    dest_a = torch.zeros(300_001, dtype=torch.bfloat16, device="cuda")
    dest_b = torch.zeros_like(dest_a)
    plain, synced = stats_tensor(cuda_device), stats_tensor(cuda_device)
    k.reduce_stats([src[0].data_ptr()], dest_a, plain, scale=scale, average=True)
    k.finalize(plain, 2.0)
    box, error = _mailbox(), torch.zeros(1, dtype=torch.int32, device="cuda")
    for epoch in (1, 2):     # two steps in a row: the flags only move forward
        k.reduce_exchange([src[0].data_ptr()], dest_b, synced, scale=scale, average=True,
                          sync=_sync([box], 0, epoch, error))
        torch.cuda.synchronize()
        assert torch.equal(dest_a.view(torch.int16), dest_b.view(torch.int16))
        for name in ("sumsq", "nonfinite", "nan", "maxabs", "norm", "found_inf"):
            i = N.STATS_FIELDS.index(name)
            assert float(synced[i]) == float(plain[i]), name
        assert int(error.item()) == 0
        assert _flag(box, N.NT_ZERO_READY, 0) == epoch and _flag(box, N.NT_ZERO_STATS, 0) == epoch


@pytest.mark.parametrize("norm_type", [2.0, float("inf")])
def test_exchange_adds_the_other_ranks_statistics_in_rank_order(cuda_device, norm_type):
    """Rank 1 of two: rank 0 has already signalled READY and STATS with its totals."""
    k = CudaShardKernels(cuda_device)
    src = _grads(2, 100_003, 2)
    dest = torch.zeros(100_003, dtype=torch.bfloat16, device="cuda")
    local = stats_tensor(cuda_device)
    k.reduce_stats([s.data_ptr() for s in src], dest.clone(), local, scale=None, average=True)
    torch.cuda.synchronize()
    mine = local.cpu().numpy()
    own, peer = _mailbox(), _mailbox()
    other = [123.25, 0.0, 0.0, 7.5]     # rank 0's {sumsq, #non-finite, #NaN, max|g|}
    epoch = 5
    _set_flag(own, N.NT_ZERO_READY, 0, epoch)
    _set_flag(own, N.NT_ZERO_STATS, 0, epoch)
    _stats_slot(own, 0).copy_(torch.tensor(other, dtype=torch.float64))
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = stats_tensor(cuda_device)
    k.reduce_exchange([s.data_ptr() for s in src], dest, out, scale=None, average=True,
                      sync=_sync([peer, own], 1, epoch, error), norm_type=norm_type)
    torch.cuda.synchronize()
    s = dict(zip(N.STATS_FIELDS, out.cpu().numpy()))
    sumsq = other[0] + mine[N.STATS_FIELDS.index("sumsq")]
    assert s["sumsq"] == sumsq
    assert s["maxabs"] == max(other[3], mine[N.STATS_FIELDS.index("maxabs")])
    assert s["found_inf"] == 0.0 and int(error.item()) == 0
    assert s["norm"] == (math.sqrt(sumsq) if norm_type == 2.0 else s["maxabs"])
    # This rank's flags and totals went to both mailboxes.
    for box in (own, peer):
        assert _flag(box, N.NT_ZERO_READY, 1) == epoch and _flag(box, N.NT_ZERO_STATS, 1) == epoch
        got = _stats_slot(box, 1).cpu().numpy()
        assert got[0] == mine[N.STATS_FIELDS.index("sumsq")] and got[3] == mine[N.STATS_FIELDS.index("maxabs")]


def test_a_rank_that_never_signals_ends_the_wait_with_an_error(cuda_device):
    k = CudaShardKernels(cuda_device)
    src = _grads(2, 50_000, 3)
    dest = torch.zeros(50_000, dtype=torch.bfloat16, device="cuda")
    out = stats_tensor(cuda_device)
    own, peer = _mailbox(), _mailbox()
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    k.reduce_exchange([s.data_ptr() for s in src], dest, out, scale=None, average=True,
                      sync=_sync([own, peer], 0, 1, error, timeout_ns=20_000_000))
    torch.cuda.synchronize()
    assert int(error.item()) & 1
    s = dict(zip(N.STATS_FIELDS, out.cpu().numpy()))
    assert s["found_inf"] == 1.0 and math.isnan(s["norm"])     # the update will skip
    assert float(torch.ones(4, device="cuda").sum()) == 4.0   # the context is still usable


def _update_exchange(grads, p0, total, *, npeers, sync, stats=None, empty=False):
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
    steps = torch.zeros(1, dtype=torch.int32, device=device)
    segs, nseg, nchunks = None, 0, 0
    if not empty:
        table, nchunks = segment_table([(grads.data_ptr(), 0, total, 0, 0)], CHUNK)
        segs, nseg = upload(table, device), 1
    peers = [torch.zeros(total, dtype=torch.bfloat16, device=device) for _ in range(npeers)]
    k.update(master=master, exp_avg=m, exp_avg_sq=v, copy=copy, grad_dtype=torch.bfloat16, segments=segs,
             num_segments=nseg, num_chunks=nchunks, steps=steps, corrections=corr.tensor, capacity=corr.capacity,
             scale=None, stats=stats, skip=stats is not None, max_norm=None, groups=[group],
             peers=[p.data_ptr() for p in peers], sync=sync)
    torch.cuda.synchronize()
    return master, copy, steps, peers


@pytest.mark.parametrize("case", ["update", "skip", "empty"])
def test_update_exchange_signals_done_after_its_pushes(cuda_device, case):
    total = 2 * CHUNK + 77
    rng = np.random.default_rng(9)
    p0 = rng.normal(0, 0.02, total).astype(np.float32)
    g = torch.from_numpy(rng.normal(0, 1e-3, total).astype(np.float32)).cuda().to(torch.bfloat16)
    own, peer = _mailbox(), _mailbox()
    epoch = 3
    _set_flag(own, N.NT_ZERO_DONE, 1, epoch)        # rank 1 has finished its step already
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    stats = None
    if case == "skip":
        stats = stats_tensor(cuda_device)
        stats[N.STATS_FIELDS.index("found_inf")] = 1.0
    master, copy, steps, peers = _update_exchange(g, p0, total, npeers=1, sync=_sync([own, peer], 0, epoch, error),
                                                  stats=stats, empty=case == "empty")
    assert int(error.item()) == 0
    for box in (own, peer):
        assert _flag(box, N.NT_ZERO_DONE, 0) == epoch
    if case == "update":
        assert int(steps[0]) == 1
        assert torch.equal(peers[0].view(torch.int16), copy.view(torch.int16))
        assert torch.equal(copy, master.to(torch.bfloat16))
    else:
        assert int(steps[0]) == 0
        assert torch.equal(master.cpu(), torch.from_numpy(p0)) and not torch.any(peers[0].float() != 0)


def test_update_exchange_timeout_sets_its_error_bit(cuda_device):
    total = CHUNK
    p0 = np.zeros(total, np.float32)
    g = torch.zeros(total, dtype=torch.bfloat16, device="cuda")
    own, peer = _mailbox(), _mailbox()
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    _update_exchange(g, p0, total, npeers=1, sync=_sync([own, peer], 0, 1, error, timeout_ns=20_000_000))
    assert int(error.item()) == 2
    assert float(torch.ones(4, device="cuda").sum()) == 4.0


def test_exchange_argument_checks(cuda_device):
    k = CudaShardKernels(cuda_device)
    src = _grads(2, 64, 4)
    dest = torch.zeros(64, dtype=torch.bfloat16, device="cuda")
    out = stats_tensor(cuda_device)
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    box = _mailbox()
    with pytest.raises(ValueError, match="mailbox 1 is NULL"):
        k.reduce_exchange([s.data_ptr() for s in src], dest, out, scale=None, average=True,
                          sync=_sync([box], 0, 1, error))
    with pytest.raises(ValueError, match="epoch and timeout_ns must be positive"):
        k.reduce_exchange([s.data_ptr() for s in src], dest, out, scale=None, average=True,
                          sync=_sync([box, box], 0, 0, error))
    with pytest.raises(ValueError, match="norm_type must be 2 or inf"):
        k.reduce_exchange([s.data_ptr() for s in src], dest, out, scale=None, average=True,
                          sync=_sync([box, box], 0, 1, error), norm_type=3.0)


def test_flag_exchange_signals_every_mailbox_and_reports_a_missing_rank(cuda_device):
    """nt_zero_flag_exchange (the READY / DONE kernel of the copy-engine pull): with the other
    rank's flag already in this rank's mailbox it returns status 0 and writes this rank's flag
    into both mailboxes; without it the wait ends after the bound with status 1 and the error
    bit of that flag (bit 0 for READY, bit 1 for DONE)."""
    k = CudaShardKernels(cuda_device)
    boxes = [_mailbox(), _mailbox()]
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    status = torch.full((1,), 7, dtype=torch.int32, device="cuda")
    _set_flag(boxes[0], N.NT_ZERO_READY, 1, 5)
    k.flag_exchange(_sync(boxes, 0, 5, error), 2, N.NT_ZERO_READY, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and int(error.item()) == 0
    assert _flag(boxes[0], N.NT_ZERO_READY, 0) == 5 and _flag(boxes[1], N.NT_ZERO_READY, 0) == 5
    k.flag_exchange(_sync(boxes, 0, 5, error, timeout_ns=20_000_000), 2, N.NT_ZERO_DONE, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 1 and int(error.item()) == 2
    assert _flag(boxes[1], N.NT_ZERO_DONE, 0) == 5
    k.flag_exchange(_sync(boxes, 0, 6, error, timeout_ns=20_000_000), 2, N.NT_ZERO_READY, status)
    torch.cuda.synchronize()
    assert int(status.item()) == 1 and int(error.item()) == 3
    assert torch.zeros(4, device="cuda").sum().item() == 0.0   # the device is still usable


def test_stats_exchange_over_piece_records_matches_the_fused_exchange(cuda_device):
    """nt_zero_stats_exchange adds the records of the shard's pieces in order and exchanges
    the totals: with one rank, the result equals the fused kernel's record for the whole
    shard up to the order of the float64 sum; with two ranks (the other's totals and STATS
    flag preset), the norm covers both; a failed READY (status 1) skips the exchange and
    reports found_inf with a NaN norm."""
    k = CudaShardKernels(cuda_device)
    count = 400_000
    src = _grads(1, count, 3)[0]
    scale = torch.tensor([1024.0], device="cuda")
    whole = stats_tensor(cuda_device)
    dest = torch.zeros(count, dtype=torch.bfloat16, device="cuda")
    k.reduce_stats([src.data_ptr()], dest, whole, scale=scale, average=True)
    k.finalize(whole, 2.0)
    pieces = [(0, 128_000), (128_000, 128_000), (256_000, 144_000)]
    records = torch.zeros((len(pieces), len(N.STATS_FIELDS)), dtype=torch.float64, device="cuda")
    for j, (off, n) in enumerate(pieces):
        k.reduce_stats([src.data_ptr() + 2 * off], dest[off:off + n], records[j], scale=scale, average=True)
    ok = torch.zeros(1, dtype=torch.int32, device="cuda")
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = stats_tensor(cuda_device)
    k.stats_exchange(records, _sync([_mailbox()], 0, 1, error), 1, ok, out)
    torch.cuda.synchronize()
    f = {name: N.STATS_FIELDS.index(name) for name in ("sumsq", "nonfinite", "nan", "maxabs", "norm", "found_inf")}
    assert abs(float(out[f["sumsq"]]) - float(whole[f["sumsq"]])) <= 1e-12 * float(whole[f["sumsq"]])
    assert abs(float(out[f["norm"]]) - float(whole[f["norm"]])) <= 1e-12 * float(whole[f["norm"]])
    for name in ("nonfinite", "nan", "maxabs", "found_inf"):
        assert float(out[f[name]]) == float(whole[f[name]]), name
    # Two ranks: the other rank's totals are already in this rank's mailbox.
    boxes = [_mailbox(), _mailbox()]
    _stats_slot(boxes[0], 1)[:] = torch.tensor([3.0, 0.0, 0.0, 0.5], dtype=torch.float64)
    _set_flag(boxes[0], N.NT_ZERO_STATS, 1, 4)
    k.stats_exchange(records, _sync(boxes, 0, 4, error), 2, ok, out)
    torch.cuda.synchronize()
    want = float(records[:, f["sumsq"]].sum().item()) + 3.0
    assert abs(float(out[f["norm"]]) - math.sqrt(want)) <= 1e-12 * math.sqrt(want)
    assert _flag(boxes[1], N.NT_ZERO_STATS, 0) == 4 and int(error.item()) == 0
    # A READY that ran out earlier in the step: no exchange, a skipped step.
    bad = torch.ones(1, dtype=torch.int32, device="cuda")
    k.stats_exchange(records, _sync(boxes, 0, 5, error), 2, bad, out)
    torch.cuda.synchronize()
    assert math.isnan(float(out[f["norm"]])) and float(out[f["found_inf"]]) == 1.0 and int(error.item()) == 1
    assert _flag(boxes[1], N.NT_ZERO_STATS, 0) == 4    # nothing was signalled


def test_flag_and_stats_exchange_reject_bad_arguments(cuda_device):
    k = CudaShardKernels(cuda_device)
    error = torch.zeros(1, dtype=torch.int32, device="cuda")
    sync = _sync([_mailbox()], 0, 1, error)
    with pytest.raises(ValueError, match="flag"):
        k.flag_exchange(sync, 1, 3)
    with pytest.raises(ValueError, match="num_ranks"):
        k.flag_exchange(sync, 9, N.NT_ZERO_READY)
    records = torch.zeros((1, len(N.STATS_FIELDS)), dtype=torch.float64, device="cuda")
    with pytest.raises(ValueError, match="norm_type"):
        k.stats_exchange(records, sync, 1, None, stats_tensor(cuda_device), norm_type=3.0)
