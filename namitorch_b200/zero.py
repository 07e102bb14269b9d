"""ZeRO-1 sharded AdamW across the GPUs of one node (one process per GPU).

The reference has no distributed code; this extends its AdamW API (namitorch/optim/adam.py)
with optimizer-state sharding. Every rank builds the same flat layout of all parameters
(64-element aligned segments, total padded to a multiple of 64 * world). Rank r owns the
contiguous shard [r*S, (r+1)*S) of that layout:

* every rank holds the full low-precision model copy (the parameters' storage) and the full
  gradient buffer (the parameters' ``.grad`` views), both in ``model_dtype``;
* rank r holds only its shard of the fp32 master weights, exp_avg and exp_avg_sq.

One step:
1. reduce-scatter the gradient buffer (NCCL, average over ranks) into the rank's shard;
2. one statistics kernel over the shard, then one all-reduce (SUM) of the 24-byte record
   {sum g^2, #non-finite, #NaN} (plus a MAX of max|g| for a non-2 norm), and a one-thread
   finalize kernel — every rank then holds the same found_inf and global norm;
3. the fused AdamW kernel over the shard's parameter pieces (unscale, skip, clip, update),
   writing the updated bf16 values into the rank's slice of the model copy;
4. all-gather of the model copy in place.

Steps 2-4 use the same C ABI entry points as the single-GPU path; a parameter cut by a
shard boundary is simply two segments on two ranks that share the same step counter value.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from . import _native as N
from .flat import ALIGN, CHUNK, FlatLayout, round_up, segment_table, span_table, stats_tensor, upload
from .optim._engine import CorrectionTable
from .optim.adam import _AmpPending, _FirstOrderAdam, _OWNERS
from .optim._common import _scalar

_SUM_FIELDS = slice(0, 3)   # sumsq, nonfinite, nan
_MAXABS = N.STATS_FIELDS.index("maxabs")
_POWSUM = N.STATS_FIELDS.index("powsum")


def shard_bounds(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of rank's shard of a layout of ``total`` elements (a multiple of world)."""
    size = total // world
    return rank * size, (rank + 1) * size


def shard_pieces(offsets: list[int], numels: list[int], start: int, stop: int) -> list[tuple[int, int, int]]:
    """(parameter index, offset within the shard, count) of every parameter piece in [start, stop)."""
    pieces = []
    for i, (off, n) in enumerate(zip(offsets, numels)):
        lo, hi = max(off, start), min(off + n, stop)
        if lo < hi:
            pieces.append((i, lo - start, hi - lo))
    return pieces


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

    def update(self, *, master, exp_avg, exp_avg_sq, copy, grad_dtype, segments, num_segments, num_chunks, steps,
               corrections, capacity, scale, stats, skip, max_norm, groups):
        group_array = (N.AdamWGroup * len(groups))(*groups)
        args = N.AdamWMtArgs(
            param=master.data_ptr(), exp_avg=exp_avg.data_ptr(), exp_avg_sq=exp_avg_sq.data_ptr(),
            model_copy=copy.data_ptr(), model_dtype=N.dtype_code(copy.dtype), grad_dtype=N.dtype_code(grad_dtype),
            segments=segments.data_ptr(), num_segments=num_segments, chunk_elems=CHUNK, num_chunks=num_chunks,
            steps=steps.data_ptr(), corrections=corrections.data_ptr(), correction_capacity=capacity,
            scale=None if scale is None else scale.data_ptr(), stats=None if stats is None else stats.data_ptr(),
            skip_nonfinite=int(skip), clip=int(max_norm is not None), max_norm=float(max_norm or 0.0),
            workspace=self.adamw_workspace.data_ptr(), error=self.error.data_ptr(), groups=group_array,
            num_groups=len(groups))
        N.call("nt_adamw_mt", N.C.byref(args), N.stream_handle())


class ZeroAdamW(_FirstOrderAdam):
    """AdamW whose fp32 state is sharded over the ranks of ``process_group``.

    Same constructor arguments as ``AdamW`` (no ``fused`` switch: always the multi-tensor
    kernel) plus ``process_group`` and ``model_dtype`` (default bfloat16). The parameters
    become views of the full model copy and their ``.grad`` views of the full gradient buffer;
    ``zero_grad`` zeroes that buffer in place."""

    _decoupled_weight_decay = True

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 1e-2,
                 *, maximize: bool = False, model_dtype=torch.bfloat16, process_group=None, average_grads: bool = True,
                 _kernels=None):
        if model_dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise TypeError("model_dtype must be torch.bfloat16, torch.float16 or torch.float32.")
        self._group = process_group
        self._average = average_grads
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
        self.params_list = params
        self.index = {id(p): i for i, p in enumerate(params)}
        base = FlatLayout.build([p.numel() for p in params])
        total = round_up(base.total, ALIGN * self.world)
        self.layout = FlatLayout(base.numels, base.offsets, total)
        self.shard_start, self.shard_stop = shard_bounds(total, self.world, self.rank)
        shard = self.shard_stop - self.shard_start
        self.pieces = shard_pieces(base.offsets, base.numels, self.shard_start, self.shard_stop)
        with torch.no_grad():
            self.copy = torch.zeros(total, dtype=self._copy_dtype, device=device)
            self.flat_grads = torch.zeros(total, dtype=self._copy_dtype, device=device)
            self.grad_shard = torch.zeros(shard, dtype=self._copy_dtype, device=device)
            self.master = torch.zeros(shard, dtype=torch.float32, device=device)
            for i, off, n in self.pieces:
                src = params[i].detach().reshape(-1)
                lo = self.shard_start + off - self.layout.offsets[i]
                self.master[off:off + n].copy_(src[lo:lo + n])
            for p, off in zip(params, self.layout.offsets):
                view = self.copy[off:off + p.numel()].view(p.shape)
                view.copy_(p.detach())
            for p, off in zip(params, self.layout.offsets):
                p.data = self.copy[off:off + p.numel()].view(p.shape)
                p.grad = self.flat_grads[off:off + p.numel()].view(p.shape)
            self.exp_avg = torch.zeros(shard, dtype=torch.float32, device=device)
            self.exp_avg_sq = torch.zeros(shard, dtype=torch.float32, device=device)
            self.steps = torch.zeros(len(params), dtype=torch.int32, device=device)
        self.corrections = CorrectionTable(device)
        self.max_step = 0
        self._reduced = False
        self._segments_key = None
        for p in params:
            _OWNERS[id(p)] = self

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
            for p, off in zip(self.params_list, self.layout.offsets):
                if p.grad is None or p.grad.data_ptr() != self.flat_grads[off:].data_ptr():
                    p.grad = self.flat_grads[off:off + p.numel()].view(p.shape)

    # ---- collectives ---------------------------------------------------------------------------
    def _adopt_foreign_grads(self):
        """Copies gradients that autograd stored outside the flat buffer back into it."""
        with torch.no_grad():
            for p, off in zip(self.params_list, self.layout.offsets):
                view = self.flat_grads[off:off + p.numel()]
                if p.grad is None:
                    view.zero_()
                    p.grad = view.view(p.shape)
                elif p.grad.data_ptr() != view.data_ptr():
                    view.copy_(p.grad.reshape(-1))
                    p.grad = view.view(p.shape)

    def _reduce(self):
        if self._reduced:
            return
        self._adopt_foreign_grads()
        op = dist.ReduceOp.AVG if self._average else dist.ReduceOp.SUM
        dist.reduce_scatter_tensor(self.grad_shard, self.flat_grads, op=op, group=self._group)
        self._reduced = True

    def _global_stats(self, scale, norm_type: float) -> torch.Tensor:
        """found_inf and the global norm, identical on every rank."""
        stats = stats_tensor(self.device)
        k = self._kernels
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
        self._reduce()
        if lazy:
            stats = self._global_stats(scale, 2.0)
            self._amp = _AmpPending(self._grad_key(self._entries()), stats, scale)
        else:
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

    def _materialize_pending(self):
        amp = self._amp
        if amp is None or (amp.scale is None and amp.max_norm is None):
            return
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
        options = self._validated_options()
        self._reduce()
        amp = self._amp
        self._amp = None
        used = sorted({gi for gi, _, _ in self._entries()})
        if len(used) > N.NT_MAX_GROUPS:
            raise RuntimeError(f"ZeroAdamW supports at most {N.NT_MAX_GROUPS} parameter groups.")
        local = {gi: k for k, gi in enumerate(used)}
        group_of = {}
        for gi, group in enumerate(self.param_groups):
            for p in group["params"]:
                group_of[self.index[id(p)]] = gi
        structs = [self._group_struct(options[gi]) for gi in used]
        self.corrections.ensure(self.max_step + 1)
        rows = [(self.grad_shard.data_ptr() + off * self.grad_shard.element_size(), off, n,
                 local[group_of[i]], i) for i, off, n in self.pieces]
        if rows:
            key = tuple(rows)
            if key != self._segments_key:
                table, nchunks = segment_table(rows, CHUNK)
                self._segments = upload(table, self.device)
                self._num_chunks = nchunks
                self._segments_key = key
            copy_shard = self.copy[self.shard_start:self.shard_stop]
            self._kernels.update(
                master=self.master, exp_avg=self.exp_avg, exp_avg_sq=self.exp_avg_sq, copy=copy_shard,
                grad_dtype=self.grad_shard.dtype, segments=self._segments, num_segments=len(rows),
                num_chunks=self._num_chunks, steps=self.steps, corrections=self.corrections.tensor,
                capacity=self.corrections.capacity, scale=None if amp is None else amp.scale,
                stats=None if amp is None else amp.stats, skip=bool(amp is not None and amp.skip),
                max_norm=None if amp is None else amp.max_norm, groups=structs)
        else:
            # A rank whose shard holds no parameter still advances the shared step counters.
            self._advance_steps_without_update(amp)
        dist.all_gather_into_tensor(self.copy, self.copy[self.shard_start:self.shard_stop], group=self._group)
        self._reduced = False
        self.max_step += 1
        return loss

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
        full = torch.empty(self.layout.total, dtype=shard.dtype, device=shard.device)
        dist.all_gather_into_tensor(full, shard, group=self._group)
        return full

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
                    for j, off, n in self.pieces:
                        if j == i:
                            lo = self.shard_start + off - self.layout.offsets[i]
                            arena[off:off + n].copy_(src[lo:lo + n])
            self.steps.copy_(torch.tensor(steps, dtype=torch.int32))
            # The model copy follows the (possibly restored) masters.
            for i, off, n in self.pieces:
                self.copy[self.shard_start + off:self.shard_start + off + n].copy_(self.master[off:off + n])
        dist.all_gather_into_tensor(self.copy, self.copy[self.shard_start:self.shard_stop].clone(), group=self._group)
        self.max_step = max(steps) if steps else 0

    @property
    def master_params(self):
        raise RuntimeError("ZeroAdamW shards its master weights; use state_dict() to assemble them.")
