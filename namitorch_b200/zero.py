"""ZeRO-1 sharded AdamW across the GPUs of one node (one process per GPU).

The reference has no distributed code; this extends its AdamW API (namitorch/optim/adam.py)
with optimizer-state sharding. Every rank builds the same flat layout of all parameters
(64-element aligned segments). The layout is cut into K pieces ("super-chunks") of N*c
elements; rank r owns slot r of every piece, i.e. the K ranges
[j*N*c + r*c, j*N*c + (r+1)*c). That ownership makes every piece contiguous across the
ranks, so both collectives run per piece on contiguous slices, in place:

* every rank holds the full low-precision model copy (the parameters' storage) and the full
  gradient buffer (the parameters' ``.grad`` views), both in ``model_dtype``;
* rank r holds only its K*c elements of the fp32 master weights, exp_avg and exp_avg_sq.

One step has two exchanges around the update, over one of two transports:

* ``transport="p2p"`` (default when every pair of GPUs can address each other's memory):
  the exchanges run inside the kernels, over NVLink, through CUDA IPC mappings of every
  rank's gradient buffer, model copy and mailbox (K = 1: one contiguous shard per rank).
  With ``exchange="flags"`` (the default) a step is two kernels and no NCCL call:
  1. ``nt_zero_reduce_scatter_exchange``: every rank signals READY into every mailbox and
     waits for everyone's (all gradients final); it pulls its shard range from every rank's
     gradient buffer, sums in f32 in rank order, writes the reduced shard and the shard's
     statistics; then it sends those statistics to every rank, waits for everyone's, adds
     them in rank order and finalizes: every rank holds the same found_inf and global norm.
     With ``pull="copy"`` the copy engines read the peers instead of the SMs: a READY
     exchange kernel, one cudaMemcpyAsync per peer and range of the shard into local staging
     on a copy stream, the same reduction per range as each range's copies land, and a
     STATS exchange kernel over the range statistics (the copy engines keep more of each
     link busy than SM loads when both directions carry data);
  2. ``nt_adamw_mt_push_exchange``: the fused AdamW kernel (unscale, skip, clip, update)
     stores each bf16 result into its own model copy and into every peer's (the
     all-gather), then signals DONE and waits for everyone's: every push has landed and
     every pull has ended.
  Every wait is bounded (``exchange_timeout``); one that runs out sets a sticky error word
  (``exchange_error`` / ``check_exchange``) and the step is skipped as for found_inf. With
  ``exchange="nccl"`` the same two kernels (without the flags) are ordered by a 4-byte NCCL
  all-reduce barrier before the pull, one SUM all-reduce of {sum g^2, #non-finite, #NaN}
  and a finalize kernel after it, and a second barrier after the push.
* ``transport="nccl"``: NCCL reduce-scatter of every piece (average over ranks), the
  statistics kernel plus the same all-reduce, then per piece the fused AdamW kernel
  followed by that piece's all-gather on a side stream, overlapping the next piece's update.

A parameter cut by a piece or rank boundary is several segments; only its last segment on a
rank advances its step counter (a negative step slot marks the others).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import _native as N
from .flat import ALIGN, CHUNK, FlatLayout, round_up, segment_table, span_table, stats_tensor, upload, zeroed_arena
from .optim._engine import CorrectionTable
from .optim.adam import _AmpPending, _FirstOrderAdam, _OWNERS
from .optim._common import _scalar

_SUM_FIELDS = slice(0, 3)   # sumsq, nonfinite, nan
_MAXABS = N.STATS_FIELDS.index("maxabs")
_POWSUM = N.STATS_FIELDS.index("powsum")


DEFAULT_PIECES = 8
COPY_PULL_PIECES = 8   # ranges of the shard in the copy-engine pull (copies of one overlap the reduction of another)


def interleaved_layout(numels: list[int], world: int, pieces: int = DEFAULT_PIECES):
    """(offsets, total, c): 64-aligned offsets of every tensor and the piece slot length c,
    with total = pieces * world * c."""
    base = FlatLayout.build(numels)
    c = round_up(-(-base.total // (pieces * world)), ALIGN)
    return base.offsets, pieces * world * c, c


def owned_ranges(world: int, rank: int, pieces: int, c: int) -> list[tuple[int, int, int]]:
    """(global start, global stop, local start) of every range rank owns."""
    return [(j * world * c + rank * c, j * world * c + (rank + 1) * c, j * c) for j in range(pieces)]


def shard_pieces(offsets: list[int], numels: list[int], ranges) -> list[tuple[int, int, int, int]]:
    """(parameter index, offset in the rank's shard, count, piece) of every owned parameter piece."""
    out = []
    for j, (start, stop, local) in enumerate(ranges):
        for i, (off, n) in enumerate(zip(offsets, numels)):
            lo, hi = max(off, start), min(off + n, stop)
            if lo < hi:
                out.append((i, local + lo - start, hi - lo, j))
    return out


class CudaShardKernels:
    """The kernel calls of one ZeRO-1 step, through libnamitorch_b200.so."""

    def __init__(self, device: torch.device):
        self.device = device
        self.workspace = torch.zeros(int(N.load().nt_grad_stats_workspace_size()), dtype=torch.uint8, device=device)
        self.adamw_workspace = torch.zeros(int(N.load().nt_adamw_workspace_size()), dtype=torch.uint8, device=device)
        self.error = torch.zeros(1, dtype=torch.int32, device=device)
        self._span_key = None
        self._spans = None

    def _span(self, buf: torch.Tensor):
        key = (buf.data_ptr(), buf.numel())
        if key != self._span_key:
            table, nchunks = span_table([key], CHUNK)
            self._spans = (upload(table, self.device), nchunks)
            self._span_key = key
        return self._spans

    def stats(self, buf, stats, *, scale, norm_type, pass_, finalize):
        spans, nchunks = self._span(buf)
        args = N.GradStatsArgs(spans=spans.data_ptr(), num_spans=1, chunk_elems=CHUNK, num_chunks=nchunks,
                               dtype=N.dtype_code(buf.dtype), scale=None if scale is None else scale.data_ptr(),
                               pass_=pass_, norm_type=float(norm_type), finalize=int(finalize),
                               stats=stats.data_ptr(), workspace=self.workspace.data_ptr(),
                               workspace_bytes=self.workspace.numel())
        N.call("nt_grad_stats", N.C.byref(args), N.stream_handle())

    def finalize(self, stats, norm_type):
        N.call("nt_grad_stats_finalize", stats.data_ptr(), float(norm_type), N.stream_handle())

    def transform(self, buf, *, scale, stats, max_norm):
        spans, nchunks = self._span(buf)
        N.call("nt_grad_transform", spans.data_ptr(), 1, CHUNK, nchunks, N.dtype_code(buf.dtype),
               None if scale is None else scale.data_ptr(), None if stats is None else stats.data_ptr(),
               int(max_norm is not None), float(max_norm or 0.0), N.stream_handle())

    def clip_value(self, buf, bound):
        spans, nchunks = self._span(buf)
        N.call("nt_grad_clip_value", spans.data_ptr(), 1, CHUNK, nchunks, N.dtype_code(buf.dtype), float(bound),
               N.stream_handle())

    def reduce_stats(self, sources, dest, stats, *, scale, average):
        """Fused reduce-scatter + pass-0 statistics over peer memory."""
        args = N.ZeroReduceArgs(num_ranks=len(sources), dtype=N.dtype_code(dest.dtype), count=dest.numel(),
                                average=int(bool(average)), dest=dest.data_ptr(),
                                scale=None if scale is None else scale.data_ptr(), stats=stats.data_ptr(),
                                workspace=self.workspace.data_ptr(), workspace_bytes=self.workspace.numel())
        for q, ptr in enumerate(sources[:N.NT_MAX_RANKS]):   # more ranks: the library rejects num_ranks
            args.sources[q] = ptr
        N.call("nt_zero_reduce_scatter_stats", N.C.byref(args), N.stream_handle())

    def reduce_exchange(self, sources, dest, stats, *, scale, average, sync, norm_type=2.0):
        """reduce_stats with the cross-GPU exchanges inside the kernel: every rank's READY before
        the pull, then every rank's shard statistics, so `stats` comes back global and final."""
        args = N.ZeroReduceArgs(num_ranks=len(sources), dtype=N.dtype_code(dest.dtype), count=dest.numel(),
                                average=int(bool(average)), dest=dest.data_ptr(),
                                scale=None if scale is None else scale.data_ptr(), stats=stats.data_ptr(),
                                workspace=self.workspace.data_ptr(), workspace_bytes=self.workspace.numel())
        for q, ptr in enumerate(sources[:N.NT_MAX_RANKS]):
            args.sources[q] = ptr
        N.call("nt_zero_reduce_scatter_exchange", N.C.byref(args), N.C.byref(sync), float(norm_type),
               N.stream_handle())

    def flag_exchange(self, sync, num_ranks, flag, status=None):
        """Signals `flag` to every rank and waits (bounded) for every rank's; `status` (int32,
        one element) records 0 or 1 (the wait ran out)."""
        N.call("nt_zero_flag_exchange", N.C.byref(sync), int(num_ranks), int(flag),
               None if status is None else status.data_ptr(), N.stream_handle())

    def stats_exchange(self, records, sync, num_ranks, ready_status, out, norm_type=2.0):
        """Adds the rows of `records` (statistics of the shard's pieces) in order, exchanges
        the totals with every rank and finalizes `out` (global and the same on every rank)."""
        N.call("nt_zero_stats_exchange", records.data_ptr(), int(records.shape[0]), N.C.byref(sync),
               int(num_ranks), None if ready_status is None else ready_status.data_ptr(), float(norm_type),
               out.data_ptr(), N.stream_handle())

    def update(self, *, master, exp_avg, exp_avg_sq, copy, grad_dtype, segments, num_segments, num_chunks, steps,
               corrections, capacity, scale, stats, skip, max_norm, groups, peers=None, schedule=None, sync=None):
        group_array = (N.AdamWGroup * len(groups))(*groups)
        args = N.AdamWMtArgs(
            param=master.data_ptr(), exp_avg=exp_avg.data_ptr(), exp_avg_sq=exp_avg_sq.data_ptr(),
            model_copy=copy.data_ptr(), model_dtype=N.dtype_code(copy.dtype), grad_dtype=N.dtype_code(grad_dtype),
            segments=None if segments is None else segments.data_ptr(), num_segments=num_segments,
            chunk_elems=CHUNK, num_chunks=num_chunks,
            steps=steps.data_ptr(), corrections=corrections.data_ptr(), correction_capacity=capacity,
            scale=None if scale is None else scale.data_ptr(), stats=None if stats is None else stats.data_ptr(),
            skip_nonfinite=int(skip), clip=int(max_norm is not None), max_norm=float(max_norm or 0.0),
            workspace=self.adamw_workspace.data_ptr(), error=self.error.data_ptr(), groups=group_array,
            num_groups=len(groups))
        if schedule is not None:
            args.lr_schedule, args.lr_schedule_rows, args.lr_schedule_columns, args.lr_step = schedule
        if sync is not None:
            array = (N.C.c_void_p * max(1, len(peers or [])))(*(peers or []))
            N.call("nt_adamw_mt_push_exchange", N.C.byref(args), array, len(peers or []), N.C.byref(sync),
                   N.stream_handle())
        elif peers:
            array = (N.C.c_void_p * len(peers))(*peers)
            N.call("nt_adamw_mt_push", N.C.byref(args), array, len(peers), N.stream_handle())
        else:
            N.call("nt_adamw_mt", N.C.byref(args), N.stream_handle())


class ZeroAdamW(_FirstOrderAdam):
    """AdamW whose fp32 state is sharded over the ranks of ``process_group``.

    Same constructor arguments as ``AdamW`` (no ``fused`` switch: always the multi-tensor
    kernel) plus ``process_group`` and ``model_dtype`` (default bfloat16). The parameters
    become views of the full model copy and their ``.grad`` views of the full gradient buffer;
    ``zero_grad`` zeroes that buffer in place."""

    _decoupled_weight_decay = True
    _sharded = True   # gradients are meaningful only after the reduce-scatter: norms and clips go through us

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 1e-2,
                 *, maximize: bool = False, model_dtype=torch.bfloat16, process_group=None, average_grads: bool = True,
                 pieces: int = DEFAULT_PIECES, transport: str = "auto", exchange: str = "flags",
                 exchange_timeout: float = 10.0, pull: str = "sm", _kernels=None):
        if model_dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise TypeError("model_dtype must be torch.bfloat16, torch.float16 or torch.float32.")
        self._group = process_group
        self._average = average_grads
        if type(pieces) is not int or pieces < 1:
            raise ValueError("pieces must be a positive integer.")
        if transport not in ("auto", "p2p", "nccl"):
            raise ValueError("transport must be 'auto', 'p2p' or 'nccl'.")
        if exchange not in ("flags", "nccl"):
            raise ValueError("exchange must be 'flags' or 'nccl'.")
        if pull not in ("sm", "copy"):
            raise ValueError("pull must be 'sm' or 'copy'.")
        if pull == "copy" and exchange != "flags":
            raise ValueError("pull='copy' orders its copies with the in-kernel flags: it needs exchange='flags'.")
        self._pull = pull
        if not (isinstance(exchange_timeout, (int, float)) and 0 < exchange_timeout <= 3600):
            raise ValueError("exchange_timeout must be a number of seconds in (0, 3600].")
        self._exchange = exchange
        self._exchange_timeout_ns = int(exchange_timeout * 1e9)
        self._epoch = 0
        self._flag_step = False
        self._mailboxes: list[int] = []
        self._pieces = pieces
        self._transport_request = transport
        self.transport = "nccl"
        self._peer_maps: list[int] = []
        self._local_stats = None
        self.timing = False
        self.last_events: list | None = None
        self._kernels = _kernels
        self._copy_dtype = model_dtype
        super().__init__(params, {"lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay,
                                  "maximize": maximize}, model_dtype=None)
        self._build()

    # ---- layout ---------------------------------------------------------------------------
    def _build(self):
        params = self._registered_parameters()
        device = params[0].device
        for p in params:
            if p.device != device:
                raise RuntimeError("ZeroAdamW parameters must live on one device per rank.")
            if p.dtype != torch.float32:
                raise RuntimeError("ZeroAdamW takes float32 parameters (they seed the fp32 master shards).")
        if self._kernels is None:
            if device.type != "cuda":
                raise RuntimeError("ZeroAdamW runs its update on CUDA devices only.")
            self._kernels = CudaShardKernels(device)
        self.world = dist.get_world_size(self._group)
        self.rank = dist.get_rank(self._group)
        self.device = device
        self.transport = self._choose_transport(device)
        if self.transport == "p2p":
            self._pieces = 1
        self.params_list = params
        self.index = {id(p): i for i, p in enumerate(params)}
        numels = [p.numel() for p in params]
        offsets, total, c = interleaved_layout(numels, self.world, self._pieces)
        self.layout = FlatLayout(numels, offsets, total)
        self.piece_len = c
        self.ranges = owned_ranges(self.world, self.rank, self._pieces, c)
        shard = self._pieces * c
        self.pieces = shard_pieces(offsets, numels, self.ranges)
        with torch.no_grad():
            self.copy = zeroed_arena(total, self._copy_dtype, device)
            self.flat_grads = zeroed_arena(total, self._copy_dtype, device)
            self.grad_shard = zeroed_arena(shard, self._copy_dtype, device)
            self.master = zeroed_arena(shard, torch.float32, device)
            for i, off, n, j in self.pieces:
                src = params[i].detach().reshape(-1)
                lo = self._global(off) - self.layout.offsets[i]
                self.master[off:off + n].copy_(src[lo:lo + n])
            for p, off in zip(params, self.layout.offsets):
                view = self.copy[off:off + p.numel()].view(p.shape)
                view.copy_(p.detach())
            views = [self.flat_grads[off:off + p.numel()].view(p.shape) for p, off in zip(params, self.layout.offsets)]
            for p, off, view in zip(params, self.layout.offsets, views):
                p.data = self.copy[off:off + p.numel()].view(p.shape)
                p.grad = view
            self.exp_avg = zeroed_arena(shard, torch.float32, device)
            self.exp_avg_sq = zeroed_arena(shard, torch.float32, device)
            self.steps = torch.zeros(len(params), dtype=torch.int32, device=device)
        # Gradient buffers: [0] is flat_grads; add_gradient_buffer adds more (double buffering).
        self.gradient_buffers = [self.flat_grads]
        self._buffer_views = [views]
        self._buffer_sources = [None]
        self._active_buffer = 0
        self.corrections = CorrectionTable(device)
        self.max_step = 0
        self._reduced = False
        self._tables = None
        self._side = torch.cuda.Stream(device) if device.type == "cuda" else None
        if self.transport == "p2p":
            self._sync = torch.zeros(1, dtype=torch.int32, device=device)
            self._mailbox = torch.zeros(N.C.sizeof(N.ZeroMailbox), dtype=torch.uint8, device=device)
            self._exchange_error = torch.zeros(1, dtype=torch.int32, device=device)
            if self._pull == "copy":
                self._build_copy_pull(shard)
            self._map_peers()
        for p in params:
            _OWNERS[id(p)] = self

    # ---- peer memory ------------------------------------------------------------------------
    def _choose_transport(self, device) -> str:
        """'p2p' when every rank's GPU can load from and store to every other rank's GPU
        (decided collectively, so all ranks agree), else 'nccl'."""
        want = self._transport_request
        if want == "nccl" or self.world == 1:
            return "nccl"
        usable = (device.type == "cuda" and isinstance(self._kernels, CudaShardKernels)
                  and dist.get_backend(self._group) == "nccl")
        devices = [None] * self.world
        dist.all_gather_object(devices, device.index if device.type == "cuda" else -1, group=self._group)
        if usable:
            try:
                usable = all(N.can_access_peer(d) for d in devices if d is not None and d >= 0)
                # The allocator's memory must be exportable (not so with expandable segments).
                probe = torch.empty(1 << 20, dtype=torch.uint8, device=device)
                N.ipc_export(probe.data_ptr())
                del probe
            except (RuntimeError, ValueError):
                usable = False
        votes = [None] * self.world
        dist.all_gather_object(votes, bool(usable), group=self._group)
        if all(votes):
            return "p2p"
        if want == "p2p":
            raise RuntimeError("ZeroAdamW(transport='p2p') needs CUDA tensors, the NCCL backend and peer access "
                               "between every pair of GPUs in the group.")
        return "nccl"

    def _map_gradient_buffer(self, buf: torch.Tensor) -> list[int]:
        """Maps every other rank's gradient buffer of the same index (a collective); returns
        the rank-ordered addresses of every rank's gradients for this rank's shard."""
        handles = [None] * self.world
        dist.all_gather_object(handles, N.ipc_export(buf.data_ptr()), group=self._group)
        grads = []
        for q, (gh, goff) in enumerate(handles):
            if q == self.rank:
                grads.append(buf.data_ptr())
                continue
            g = N.ipc_open(gh, goff)
            self._peer_maps.append(g)
            grads.append(g)
        shard_bytes = self.rank * self.piece_len * buf.element_size()
        return [g + shard_bytes for g in grads]

    def _map_peers(self):
        """Maps every other rank's gradient buffer and model copy into this process."""
        self._sources = self._map_gradient_buffer(self.flat_grads)
        self._buffer_sources[0] = self._sources
        handles = [None] * self.world
        dist.all_gather_object(handles, N.ipc_export(self.copy.data_ptr()), group=self._group)
        copies = []
        for q, (ch, coff) in enumerate(handles):
            if q == self.rank:
                copies.append(self.copy.data_ptr())
                continue
            c = N.ipc_open(ch, coff)
            self._peer_maps.append(c)
            copies.append(c)
        shard_bytes = self.rank * self.piece_len * self.copy.element_size()
        # Where this rank's shard lands in every other rank's copy, addressed like the local
        # copy base (the kernel adds the shard-local offset).
        self._push = [c + shard_bytes for q, c in enumerate(copies) if q != self.rank]
        # Every rank's mailbox (the in-kernel exchanges write epochs and statistics there).
        handles = [None] * self.world
        dist.all_gather_object(handles, N.ipc_export(self._mailbox.data_ptr()), group=self._group)
        self._mailboxes = []
        for q, (mh, moff) in enumerate(handles):
            if q == self.rank:
                self._mailboxes.append(self._mailbox.data_ptr())
                continue
            m = N.ipc_open(mh, moff)
            self._peer_maps.append(m)
            self._mailboxes.append(m)
        dist.barrier(group=self._group)

    def _build_copy_pull(self, shard: int) -> None:
        """State of the copy-engine pull: one staging buffer per peer for this rank's shard,
        the shard cut into COPY_PULL_PIECES ranges (64-element multiples) so that the local
        reduction of one range runs while the copies of the next are in flight, one
        statistics record per range, and a copy stream with one event per range."""
        with torch.no_grad():
            self._staging = zeroed_arena(max(self.world - 1, 1) * shard, self._copy_dtype, self.device)
        step = round_up(-(-shard // COPY_PULL_PIECES), ALIGN)
        self._pull_ranges = [(off, min(step, shard - off)) for off in range(0, shard, step)]
        self._records = torch.zeros((len(self._pull_ranges), len(N.STATS_FIELDS)), dtype=torch.float64,
                                    device=self.device)
        self._ready_status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._copy_stream = torch.cuda.Stream(self.device)
        self._pull_events = [torch.cuda.Event() for _ in self._pull_ranges]

    def _pull_by_copy(self, scale, stats) -> None:
        """The reduce-scatter with copy-engine reads: READY to and from every rank; the peers'
        contributions to this rank's shard copied range by range into local staging (one
        cudaMemcpyAsync per peer and range, on the copy stream); each range reduced in rank
        order with its statistics as soon as its copies land; then the statistics exchange
        over the range records. Every rank's gradients are read only after its READY, and
        this rank's STATS follows the end of its copies, so the closing DONE exchange still
        means that no peer reads this rank's gradients any more."""
        k = self._kernels
        sync = self._sync_args()
        compute = torch.cuda.current_stream(self.device)
        k.flag_exchange(sync, self.world, N.NT_ZERO_READY, self._ready_status)
        self._copy_stream.wait_stream(compute)
        esize = self.flat_grads.element_size()
        shard = self.grad_shard.numel()
        base = self._staging.data_ptr()
        slot = {q: i for i, q in enumerate(q for q in range(self.world) if q != self.rank)}
        handle = N.stream_handle(self._copy_stream)
        for (off, n), event in zip(self._pull_ranges, self._pull_events):
            for q, i in slot.items():
                N.call("nt_memcpy_async", base + (i * shard + off) * esize, self._sources[q] + off * esize,
                       n * esize, handle)
            event.record(self._copy_stream)
        for j, ((off, n), event) in enumerate(zip(self._pull_ranges, self._pull_events)):
            compute.wait_event(event)
            sources = [self._sources[q] + off * esize if q == self.rank else base + (slot[q] * shard + off) * esize
                       for q in range(self.world)]
            k.reduce_stats(sources, self.grad_shard[off:off + n], self._records[j], scale=scale,
                           average=self._average)
        k.stats_exchange(self._records, sync, self.world, self._ready_status, stats)

    def _uses_flags(self) -> bool:
        return self.transport == "p2p" and self._exchange == "flags"

    def _sync_args(self) -> "N.ZeroSync":
        sync = N.ZeroSync(rank=self.rank, epoch=self._epoch, timeout_ns=self._exchange_timeout_ns,
                          error=self._exchange_error.data_ptr())
        for q, ptr in enumerate(self._mailboxes):
            sync.mailboxes[q] = ptr
        return sync

    def exchange_error(self) -> int:
        """The in-kernel exchanges' sticky error word (synchronises): bit 0 = a wait of the
        reduce-scatter ran out (that step was skipped as if found_inf), bit 1 = the update's
        closing wait ran out. 0 over NCCL or when every wait completed."""
        if not self._uses_flags():
            return 0
        return int(self._exchange_error.item())

    def check_exchange(self) -> None:
        """Raises RuntimeError if any in-kernel wait on another rank has run out."""
        code = self.exchange_error()
        if code:
            raise RuntimeError(f"ZeroAdamW: a wait on another rank ran out (error word {code:#x}); a rank stopped "
                               "or fell more than exchange_timeout behind.")

    def add_gradient_buffer(self) -> int:
        """Allocates one more full gradient buffer on every rank (a collective call) and, over
        the p2p transport, maps the peers' buffers of the same index. Returns the index for
        ``use_gradient_buffer``: a data loader can fill one buffer while a step reduces the
        other."""
        with torch.no_grad():
            buf = zeroed_arena(self.flat_grads.numel(), self.flat_grads.dtype, self.device)
        self.gradient_buffers.append(buf)
        self._buffer_views.append([buf[off:off + p.numel()].view(p.shape)
                                   for p, off in zip(self.params_list, self.layout.offsets)])
        self._buffer_sources.append(self._map_gradient_buffer(buf) if self.transport == "p2p" else None)
        if self.transport == "p2p":
            dist.barrier(group=self._group)
        return len(self.gradient_buffers) - 1

    def use_gradient_buffer(self, index: int) -> None:
        """Makes gradient buffer `index` the one the next step reduces; the parameters' ``.grad``
        become its views. Every rank must select the same index for a step."""
        if self._reduced:
            raise RuntimeError("use_gradient_buffer cannot switch buffers in the middle of a step.")
        self._active_buffer = index
        self.flat_grads = self.gradient_buffers[index]
        if self._buffer_sources[index] is not None:
            self._sources = self._buffer_sources[index]
        for p, view in zip(self.params_list, self._buffer_views[index]):
            p.grad = view

    def close(self) -> None:
        """Unmaps the peers' buffers (collective with the other ranks' close())."""
        if self._peer_maps:
            torch.cuda.synchronize(self.device)
            for ptr in self._peer_maps:
                N.ipc_close(ptr)
            self._peer_maps = []

    def _barrier(self):
        """Stream-ordered: later work on this stream starts after every rank reached it."""
        dist.all_reduce(self._sync, op=dist.ReduceOp.MAX, group=self._group)

    def _global(self, local: int) -> int:
        """Global flat offset of an element of the rank's shard."""
        j, r = divmod(local, self.piece_len)
        return j * self.world * self.piece_len + self.rank * self.piece_len + r

    def _piece_slices(self, j: int):
        n, c = self.world, self.piece_len
        full = slice(j * n * c, (j + 1) * n * c)
        mine = slice(j * n * c + self.rank * c, j * n * c + (self.rank + 1) * c)
        return full, mine

    def _event(self):
        if self.timing and self.device.type == "cuda":
            e = torch.cuda.Event(enable_timing=True)
            e.record()
            self.last_events.append(e)

    def _ensure_engine(self):
        return self

    def _uses_engine(self) -> bool:
        return True

    @property
    def flat_gradient_buffer(self) -> torch.Tensor:
        return self.flat_grads

    def zero_grad(self, set_to_none: bool = True) -> None:
        if type(set_to_none) is not bool:
            raise TypeError("set_to_none must be a Python bool.")
        with torch.no_grad():
            self.flat_grads.zero_()
            for p, own in zip(self.params_list, self._buffer_views[self._active_buffer]):
                if p.grad is not own:
                    p.grad = own

    # ---- collectives ---------------------------------------------------------------------------
    def _adopt_foreign_grads(self):
        """Copies gradients that autograd stored outside the flat buffer back into it."""
        with torch.no_grad():
            for p, own in zip(self.params_list, self._buffer_views[self._active_buffer]):
                if p.grad is own:
                    continue
                if p.grad is None:
                    own.zero_()
                elif p.grad.data_ptr() != own.data_ptr():
                    own.view(-1).copy_(p.grad.reshape(-1))
                p.grad = own

    def _reduce(self, scale=None):
        """Reduce-scatters the gradients (once per step). Over p2p the statistics of g / scale
        come out of the same kernel and are kept for _global_stats: already global and final
        with the in-kernel exchange, the shard's own with NCCL ordering."""
        if self._reduced:
            return
        self._adopt_foreign_grads()
        if self.timing:
            self.last_events = []
        self._event()
        if self.transport == "p2p":
            stats = stats_tensor(self.device)
            if self._uses_flags():
                # READY, the pull, the statistics exchange and the finalize: the record comes
                # back global (the same on every rank). With pull='sm' all of it is one
                # kernel; with pull='copy' the copy engines read the peers.
                self._epoch += 1
                if self._pull == "copy":
                    self._pull_by_copy(scale, stats)
                else:
                    self._kernels.reduce_exchange(self._sources, self.grad_shard, stats, scale=scale,
                                                  average=self._average, sync=self._sync_args())
                self._local_stats = (scale, stats, True)
                self._flag_step = True
            else:
                self._barrier()
                self._kernels.reduce_stats(self._sources, self.grad_shard, stats, scale=scale, average=self._average)
                self._local_stats = (scale, stats, False)
            self._event()
            self._reduced = True
            return
        op = dist.ReduceOp.AVG if self._average else dist.ReduceOp.SUM
        c = self.piece_len
        for j in range(self._pieces):
            full, _ = self._piece_slices(j)
            dist.reduce_scatter_tensor(self.grad_shard[j * c:(j + 1) * c], self.flat_grads[full], op=op,
                                       group=self._group)
        self._event()
        self._reduced = True

    def _global_stats(self, scale, norm_type: float) -> torch.Tensor:
        """found_inf and the global norm, identical on every rank."""
        k = self._kernels
        cached, self._local_stats = self._local_stats, None
        if cached is not None and cached[0] is scale and cached[2]:
            # Global already (the in-kernel exchange). p = 2 is final; inf only needs the
            # finalize of the global max; any other p a second pass and one all-reduce.
            stats = cached[1]
            if norm_type == 2.0:
                return stats
            stats = stats.clone()
            if norm_type != float("inf"):
                k.stats(self.grad_shard, stats, scale=scale, norm_type=norm_type, pass_=1, finalize=False)
                dist.all_reduce(stats[_POWSUM:_POWSUM + 1], op=dist.ReduceOp.SUM, group=self._group)
            k.finalize(stats, norm_type)
            return stats
        if cached is not None and cached[0] is scale:
            stats = cached[1]          # pass 0 ran inside the p2p reduce-scatter
        else:
            stats = stats_tensor(self.device)
            k.stats(self.grad_shard, stats, scale=scale, norm_type=norm_type, pass_=0, finalize=False)
        dist.all_reduce(stats[_SUM_FIELDS], op=dist.ReduceOp.SUM, group=self._group)
        if norm_type != 2.0:
            dist.all_reduce(stats[_MAXABS:_MAXABS + 1], op=dist.ReduceOp.MAX, group=self._group)
        if not (norm_type == 2.0 or norm_type == float("inf")):
            k.stats(self.grad_shard, stats, scale=scale, norm_type=norm_type, pass_=1, finalize=False)
            dist.all_reduce(stats[_POWSUM:_POWSUM + 1], op=dist.ReduceOp.SUM, group=self._group)
        k.finalize(stats, norm_type)
        return stats

    # ---- hooks used by GradScaler / clip_grad_norm_ -----------------------------------------
    def _entries(self):
        index = {id(group): k for k, group in enumerate(self.param_groups)}
        return [(index[id(group)], p, p.grad) for group in self.param_groups for p in group["params"]]

    def _amp_gradients(self):
        return [self.grad_shard]

    def _amp_unscale_(self, scale: torch.Tensor, lazy: bool) -> torch.Tensor:
        self._reduce(scale if lazy else None)
        if lazy:
            stats = self._global_stats(scale, 2.0)
            self._amp = _AmpPending(self._grad_key(self._entries()), stats, scale)
        else:
            self._local_stats = None
            self._kernels.transform(self.grad_shard, scale=scale, stats=None, max_norm=None)
            stats = self._global_stats(None, 2.0)
            self._amp = _AmpPending(self._grad_key(self._entries()), stats, None)
        return stats

    def _lazy_clip(self, max_norm: float, norm_type: float, check=None):
        self._reduce()
        amp = self._amp
        if amp is not None and amp.max_norm is not None:
            self._materialize_pending()
            amp = self._amp
        if amp is not None and norm_type == 2.0:
            stats = amp.stats
        else:
            stats = self._global_stats(None if amp is None else amp.scale, norm_type)
            if amp is not None:
                merged = amp.stats.clone()
                merged[N.STATS_FIELDS.index("norm")] = stats[N.STATS_FIELDS.index("norm")]
                stats = merged
        if check is not None:
            check(stats)
        if amp is None:
            amp = _AmpPending(self._grad_key(self._entries()), stats, None)
        else:
            amp.stats = stats
        amp.max_norm = float(max_norm)
        self._amp = amp
        return stats

    def _grad_norm(self, norm_type: float) -> torch.Tensor:
        """Global statistics of the reduced gradients as the next step would see them
        (get_grad_norm on this optimizer's parameters)."""
        self._reduce()
        amp = self._amp
        if amp is not None and amp.max_norm is not None:
            self._materialize_pending()
            amp = self._amp
        return self._global_stats(None if amp is None else amp.scale, norm_type)

    def _clip_value_(self, bound: float) -> None:
        """clip_grad_value_ on this optimizer's parameters: clamps the reduced shard."""
        self._reduce()
        self._materialize_pending()
        self._local_stats = None
        self._kernels.clip_value(self.grad_shard, bound)

    def _materialize_pending(self):
        amp = self._amp
        if amp is None or (amp.scale is None and amp.max_norm is None):
            return
        self._local_stats = None
        self._kernels.transform(self.grad_shard, scale=amp.scale, stats=amp.stats, max_norm=amp.max_norm)
        amp.scale = None
        amp.max_norm = None

    # ---- step ---------------------------------------------------------------------------------
    def step(self, closure=None):
        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            raise RuntimeError("Optimizer steps are not allowed during CUDA graph capture.")
        if closure is not None and not callable(closure):
            raise TypeError("Optimizer closure must be callable or None.")
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        self._reduce()
        amp = self._amp
        self._amp = None
        structs, tables = self._update_plan()
        self._event()
        cuda = self.device.type == "cuda"
        main = torch.cuda.current_stream(self.device) if cuda else None
        self._local_stats = None
        if self.transport == "p2p":
            if self._flag_step:
                # The update and push, then DONE to every rank and a wait for everyone's, in one
                # kernel (launched even for an empty shard, which only takes part in DONE).
                self._launch_update(tables[0], structs, amp, 0, self._push, sync=self._sync_args())
                self._flag_step = False
                self._event()
            else:
                self._launch_update(tables[0], structs, amp, 0, self._push)
                self._event()
                self._barrier()
            self._event()
            if not self.pieces:
                self._advance_steps_without_update(amp)
            self._event()
            self._reduced = False
            self.max_step += 1
            return loss
        if cuda:
            self._side.wait_stream(main)
        for j in range(self._pieces):
            self._launch_update(tables[j], structs, amp, j, None)
            full, mine = self._piece_slices(j)
            if cuda:
                # The piece's all-gather overlaps the next piece's update.
                self._side.wait_stream(main)
                with torch.cuda.stream(self._side):
                    dist.all_gather_into_tensor(self.copy[full], self.copy[mine], group=self._group)
            else:
                dist.all_gather_into_tensor(self.copy[full], self.copy[mine], group=self._group)
        self._event()
        if cuda:
            main.wait_stream(self._side)
        if not self.pieces:
            # A rank whose shard holds no parameter still advances the shared step counters.
            self._advance_steps_without_update(amp)
        self._event()
        self._reduced = False
        self.max_step += 1
        return loss

    def _update_plan(self):
        """(group coefficient structs, per-piece segment tables) for the next update."""
        options = self._validated_options()
        used = sorted({gi for gi, _, _ in self._entries()})
        if len(used) > N.NT_MAX_GROUPS:
            raise RuntimeError(f"ZeroAdamW supports at most {N.NT_MAX_GROUPS} parameter groups.")
        local = {gi: k for k, gi in enumerate(used)}
        structs = [self._group_struct(options[gi]) for gi in used]
        for gi, st in zip(used, structs):
            st.schedule_column = gi
        self.corrections.ensure(self.max_step + 1)
        return structs, self._piece_tables(local)

    def _launch_update(self, table, structs, amp, j: int, peers, sync=None):
        """The fused AdamW kernel over piece j of the shard (pushing into `peers` if given; with
        `sync`, closing the step with the in-kernel DONE exchange, even with no segments)."""
        if table is None:
            if sync is None:
                return
            table = (None, 0, 0)
        scheduler = getattr(self, "_lr_schedule", None)
        schedule = None if scheduler is None else scheduler._schedule_args()
        segs, nseg, nchunks = table
        self._kernels.update(
            master=self.master, exp_avg=self.exp_avg, exp_avg_sq=self.exp_avg_sq, copy=self._copy_base(j),
            grad_dtype=self.grad_shard.dtype, segments=segs, num_segments=nseg, num_chunks=nchunks,
            steps=self.steps, corrections=self.corrections.tensor, capacity=self.corrections.capacity,
            scale=None if amp is None else amp.scale, stats=None if amp is None else amp.stats,
            skip=bool(amp is not None and amp.skip), max_norm=None if amp is None else amp.max_norm,
            groups=structs, peers=peers, **({"schedule": schedule} if schedule is not None else {}),
            **({"sync": sync} if sync is not None else {}))

    def benchmark_shard_update(self, iters: int) -> float:
        """Mean device time (ms) of the shard's AdamW update alone -- no reduce-scatter, no
        statistics, no all-gather or push -- over `iters` launches. It advances the optimizer
        state like that many un-scaled, un-clipped steps on the current reduced gradients, so
        call it only when the state no longer matters (a benchmark's last phase)."""
        structs, tables = self._update_plan()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        for j in range(self._pieces):
            self._launch_update(tables[j], structs, None, j, None)
        start.record()
        for _ in range(iters):
            for j in range(self._pieces):
                self._launch_update(tables[j], structs, None, j, None)
        end.record()
        end.synchronize()
        return start.elapsed_time(end) / iters

    def _copy_base(self, j: int) -> torch.Tensor:
        """The model copy as the kernel addresses it for piece j: the kernel writes element
        `local` (shard offset, in [j*c, (j+1)*c)) at base + local, and that element's global
        position is local + j*(N-1)*c + r*c."""
        return self.copy[j * (self.world - 1) * self.piece_len + self.rank * self.piece_len:]

    def _piece_tables(self, local_group):
        """One segment table per piece; the copy pointer offset is folded into each segment."""
        key = (tuple(local_group.items()),)
        if self._tables is not None and self._tables[0] == key:
            return self._tables[1]
        group_of = {}
        for gi, group in enumerate(self.param_groups):
            for p in group["params"]:
                group_of[self.index[id(p)]] = gi
        last_piece = {}
        for i, off, n, j in self.pieces:
            last_piece[i] = max(last_piece.get(i, -1), j)
        esize = self.grad_shard.element_size()
        tables = []
        for j in range(self._pieces):
            rows = []
            for i, off, n, jj in self.pieces:
                if jj != j:
                    continue
                slot = i if last_piece[i] == j else -i - 1
                rows.append((self.grad_shard.data_ptr() + off * esize, off, n, local_group[group_of[i]], slot))
            if not rows:
                tables.append(None)
                continue
            table, nchunks = segment_table(rows, CHUNK)
            tables.append((upload(table, self.device), len(rows), nchunks))
        self._tables = (key, tables)
        return tables

    def _advance_steps_without_update(self, amp):
        if amp is not None and amp.skip:
            inc = (amp.stats[N.STATS_FIELDS.index("found_inf")] == 0).to(torch.int32)
            self.steps += inc
        else:
            self.steps += 1

    def _group_struct(self, options):
        lr = options["lr"]
        beta1, beta2 = options["betas"]
        wd = options["weight_decay"]
        return N.AdamWGroup(
            lr=float(_scalar(lr)), beta1=float(_scalar(beta1)), beta2=float(_scalar(beta2)),
            one_minus_beta1=float(_scalar(1 - beta1)), one_minus_beta2=float(_scalar(1 - beta2)),
            eps=float(_scalar(options["eps"], "eps")), weight_decay=float(_scalar(wd)),
            decay_factor=float(_scalar(1 - lr * wd, "decay factor")), maximize=int(bool(options["maximize"])),
            decay_mode=N.NT_DECAY_NONE if wd == 0 else N.NT_DECAY_DECOUPLED, update_parameter=int(lr != 0),
            correction_row=self.corrections.row(beta1, beta2))

    # ---- state ----------------------------------------------------------------------------------
    def _gather_shards(self, shard: torch.Tensor) -> torch.Tensor:
        """Every rank's shard, reassembled in the global (interleaved) layout."""
        gathered = torch.empty(self.layout.total, dtype=shard.dtype, device=shard.device)
        dist.all_gather_into_tensor(gathered, shard, group=self._group)
        # gathered is [rank][piece][c]; the layout is [piece][rank][c].
        return gathered.view(self.world, self._pieces, self.piece_len).transpose(0, 1).reshape(-1)

    def _state_by_id(self):
        exported = self._full_state()
        return {id(p): st for p, st in zip(self.params_list, exported) if st is not None}

    def _full_state(self):
        """Per-parameter state assembled from every shard (a collective: call on all ranks).

        A rank only advances the counters of parameters inside its shard; counters never
        decrease, so the maximum over ranks is the owner's value."""
        counters = self.steps.clone()
        dist.all_reduce(counters, op=dist.ReduceOp.MAX, group=self._group)
        steps = counters.cpu().tolist()
        m = self._gather_shards(self.exp_avg)
        v = self._gather_shards(self.exp_avg_sq)
        master = self._gather_shards(self.master)
        out = []
        for i, (p, off) in enumerate(zip(self.params_list, self.layout.offsets)):
            if steps[i] == 0:
                out.append(None)
                continue
            n = p.numel()
            out.append({"step": int(steps[i]), "exp_avg": m[off:off + n].view(p.shape).clone(),
                        "exp_avg_sq": v[off:off + n].view(p.shape).clone(),
                        "master_param": master[off:off + n].view(p.shape).clone()})
        return out

    def _allowed_state_fields(self):
        return {"step", "exp_avg", "exp_avg_sq", "master_param"}

    def _export_state(self, parameters):
        indices = {id(p): k for k, p in enumerate(parameters)}
        full = self._full_state()
        return {indices[id(p)]: st for p, st in zip(self.params_list, full) if st is not None}

    def _import_state(self, index_to_parameter, saved_state):
        steps = [0] * len(self.params_list)
        with torch.no_grad():
            self.exp_avg.zero_()
            self.exp_avg_sq.zero_()
            for index, values in saved_state.items():
                parameter = index_to_parameter[index]
                self._check_state(values, parameter, f"state[{index}]")
                if not values:
                    continue
                i = self.index[id(parameter)]
                steps[i] = int(values["step"])
                for name, arena in (("exp_avg", self.exp_avg), ("exp_avg_sq", self.exp_avg_sq),
                                    ("master_param", self.master)):
                    if name not in values:
                        continue
                    src = values[name]
                    src = torch.from_numpy(src) if isinstance(src, np.ndarray) else src
                    src = src.detach().reshape(-1).to(device=self.device, dtype=torch.float32)
                    for k, off, n, j in self.pieces:
                        if k == i:
                            lo = self._global(off) - self.layout.offsets[i]
                            arena[off:off + n].copy_(src[lo:lo + n])
            self.steps.copy_(torch.tensor(steps, dtype=torch.int32))
            # The model copy follows the (possibly restored) masters.
            for k, off, n, j in self.pieces:
                g = self._global(off)
                self.copy[g:g + n].copy_(self.master[off:off + n])
        for j in range(self._pieces):
            full, mine = self._piece_slices(j)
            dist.all_gather_into_tensor(self.copy[full], self.copy[mine].clone(), group=self._group)
        self.max_step = max(steps) if steps else 0

    @property
    def master_params(self):
        raise RuntimeError("ZeroAdamW shards its master weights; use state_dict() to assemble them.")
