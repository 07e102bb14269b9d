"""Device state of a multi-tensor Adam / AdamW optimizer.

One engine owns, for the parameters of one optimizer on one CUDA device:
* flat fp32 arenas for the master weights, exp_avg and exp_avg_sq (FlatLayout offsets);
* optionally a bf16 / fp16 model-copy arena — the parameters the model computes with;
* one int32 step counter per parameter on the device (``state["step"]``), advanced by the
  update kernel itself so that a GradScaler skip never needs a host round trip;
* the bias-correction table f32(1 - beta^t) computed on the host with the reference's
  own expression (namitorch/optim/adam.py:38-39 and :85);
* cached device segment tables, re-uploaded only when gradient storage moves.
"""
from __future__ import annotations

import numpy as np
import torch

from .. import _native as N
from ..flat import CHUNK, FlatLayout, segment_table, upload, zeroed_arena
from ._common import _scalar


class CorrectionTable:
    """Rows of (f32(1 - beta1^t), f32(1 - beta2^t)) for t = 0 .. capacity-1, one row per (beta1, beta2)."""

    def __init__(self, device: torch.device):
        self.device = device
        self.rows: list[tuple[float, float]] = []
        self.host: list[np.ndarray] = []
        self.capacity = 0
        self.tensor: torch.Tensor | None = None
        self._dirty = True

    @staticmethod
    def _entries(beta1: float, beta2: float, start: int, stop: int) -> np.ndarray:
        out = np.empty((stop - start, 2), np.float32)
        for k, t in enumerate(range(start, stop)):
            out[k, 0] = _scalar(1 - beta1 ** t)
            out[k, 1] = _scalar(1 - beta2 ** t)
        return out

    def row(self, beta1: float, beta2: float) -> int:
        key = (float(beta1), float(beta2))
        if key in self.rows:
            return self.rows.index(key)
        self.rows.append(key)
        self.host.append(self._entries(key[0], key[1], 0, self.capacity))
        self._dirty = True
        return len(self.rows) - 1

    def saturated(self) -> bool:
        return self.capacity > 1 and all(bool(np.all(h[-1] == np.float32(1.0))) for h in self.host)

    def ensure(self, max_step: int) -> None:
        """Makes every step t <= max_step readable (directly, or through a saturated last row)."""
        need = int(max_step) + 1
        if self.capacity < need and not self.saturated():
            new_capacity = max(need + 256, 2 * self.capacity, 1024)
            for i, (b1, b2) in enumerate(self.rows):
                self.host[i] = np.concatenate([self.host[i], self._entries(b1, b2, self.capacity, new_capacity)])
            self.capacity = new_capacity
            self._dirty = True
        if self._dirty:
            table = np.stack(self.host) if self.host else np.zeros((1, max(self.capacity, 2), 2), np.float32)
            self.tensor = torch.from_numpy(np.ascontiguousarray(table)).to(self.device)
            self._dirty = False


class FusedAdamEngine:
    def __init__(self, params: list[torch.Tensor], *, model_dtype: torch.dtype | None = None):
        if not params:
            raise ValueError("Optimizer cannot receive an empty parameter list.")
        device = params[0].device
        for p in params:
            if p.device.type != "cuda":
                raise RuntimeError(
                    "namitorch_b200 runs the optimizer step on CUDA only; move the parameters to a CUDA device "
                    f"first (got {p.device}).")
            if p.device != device:
                raise RuntimeError(f"Operands are on different devices: {device}, {p.device}; "
                                   "use an explicit .to() transfer.")
            if p.dtype != torch.float32:
                raise RuntimeError(
                    "fused=True requires non-overlapping contiguous float32 CUDA parameters, gradients and states "
                    f"on the same device (got {p.dtype}).")
        if model_dtype not in (None, torch.float16, torch.bfloat16):
            raise TypeError("model_dtype must be None, torch.float16 or torch.bfloat16.")
        N.load()
        self.device = device
        self.params = list(params)
        self.index = {id(p): i for i, p in enumerate(self.params)}
        self.layout = FlatLayout.build([p.numel() for p in self.params])
        self.model_dtype = model_dtype
        total = self.layout.total
        with torch.no_grad(), torch.cuda.device(device):
            self.master = zeroed_arena(total, torch.float32, device)
            for p, off in zip(self.params, self.layout.offsets):
                self.master[off:off + p.numel()].copy_(p.detach().reshape(-1))
            if model_dtype is not None:
                self.copy = zeroed_arena(total, model_dtype, device)
                N.call("nt_cast", self.copy.data_ptr(), N.dtype_code(model_dtype), self.master.data_ptr(),
                       N.NT_F32, total, N.stream_handle())
            else:
                self.copy = None
            for p, off in zip(self.params, self.layout.offsets):
                arena = self.copy if self.copy is not None else self.master
                if p.grad is not None and (p.grad.dtype != arena.dtype):
                    p.grad = None
                p.data = arena[off:off + p.numel()].view(p.shape)
            self.exp_avg: torch.Tensor | None = None
            self.exp_avg_sq: torch.Tensor | None = None
            self.steps = torch.zeros(len(self.params), dtype=torch.int32, device=device)
            self.workspace = torch.zeros(int(N.load().nt_adamw_workspace_size()), dtype=torch.uint8, device=device)
            self.error = torch.zeros(1, dtype=torch.int32, device=device)
        self.loaded: set[int] = set()
        self.max_step = 0
        self.corrections = CorrectionTable(device)
        # Device segment tables by (gradient address, offset, count, group, index) rows: a few
        # are kept, so gradients that alternate between buffers (double-buffered host
        # copies) find their table without a new upload.
        self._segment_tables: dict[tuple, tuple[torch.Tensor, int, int]] = {}
        self._segments = None
        self._num_segments = 0
        self._num_chunks = 0

    # ---- views ------------------------------------------------------------------------------
    def view(self, arena: torch.Tensor, i: int) -> torch.Tensor:
        p = self.params[i]
        off = self.layout.offsets[i]
        return arena[off:off + p.numel()].view(p.shape)

    def master_view(self, i: int) -> torch.Tensor:
        return self.view(self.master, i)

    def ensure_moments(self) -> None:
        if self.exp_avg is None:
            with torch.cuda.device(self.device):
                self.exp_avg = zeroed_arena(self.master.numel(), torch.float32, self.device)
                self.exp_avg_sq = zeroed_arena(self.master.numel(), torch.float32, self.device)

    @property
    def grad_dtype(self) -> torch.dtype:
        return self.model_dtype if self.model_dtype is not None else torch.float32

    # ---- the fused step ---------------------------------------------------------------------
    def group_struct(self, options: dict, decoupled: bool) -> N.AdamWGroup:
        lr = options["lr"]
        beta1, beta2 = options["betas"]
        wd = options["weight_decay"]
        if wd == 0:
            mode = N.NT_DECAY_NONE
        else:
            mode = N.NT_DECAY_DECOUPLED if decoupled else N.NT_DECAY_COUPLED
        decay = _scalar(1 - lr * wd, "decay factor") if decoupled else np.float32(1.0)
        return N.AdamWGroup(
            lr=float(_scalar(lr)), beta1=float(_scalar(beta1)), beta2=float(_scalar(beta2)),
            one_minus_beta1=float(_scalar(1 - beta1)), one_minus_beta2=float(_scalar(1 - beta2)),
            eps=float(_scalar(options["eps"], "eps")), weight_decay=float(_scalar(wd)), decay_factor=float(decay),
            maximize=int(bool(options["maximize"])), decay_mode=mode, update_parameter=int(lr != 0),
            correction_row=self.corrections.row(beta1, beta2))

    def step(self, entries: list[tuple[int, torch.Tensor, torch.Tensor]], group_options: list[dict], *,
             decoupled: bool, scale: torch.Tensor | None = None, stats: torch.Tensor | None = None,
             skip_nonfinite: bool = False, max_norm: float | None = None, schedule=None) -> None:
        """One update of every (group index, parameter, gradient) entry. `schedule` is a
        device learning-rate schedule (table, rows, columns, step pointer) or None."""
        if not entries:
            return
        self.ensure_moments()
        used = sorted({gi for gi, _, _ in entries})
        for start in range(0, len(used), N.NT_MAX_GROUPS):
            batch = used[start:start + N.NT_MAX_GROUPS]
            local = {gi: k for k, gi in enumerate(batch)}
            structs = [self.group_struct(group_options[gi], decoupled) for gi in batch]
            for gi, st in zip(batch, structs):
                st.schedule_column = gi
            selected = entries if len(batch) == len(used) else [e for e in entries if e[0] in local]
            self._launch(selected, local, structs, scale, stats, skip_nonfinite, max_norm, schedule)
        self.max_step += 1

    def _launch(self, entries, local, structs, scale, stats, skip_nonfinite, max_norm, schedule=None) -> None:
        self.corrections.ensure(self.max_step + 1)
        keep = []
        # The segment table depends on the entries, their group mapping and every gradient's
        # address; the addresses are swept every step (a gradient whose storage moved gets a
        # new table), the rest is compared by identity.
        fast_key = (id(entries), tuple(local.items()), tuple(map(torch.Tensor.data_ptr, (g for _, _, g in entries))))
        cached = self.__dict__.get("_rows_cache")
        if cached is None or cached[0] != fast_key or cached[1] is not entries:
            rows = []
            contiguous = True
            for gi, p, g in entries:
                i = self.index[id(p)]
                if not g.is_contiguous():
                    g = g.contiguous()
                    keep.append(g)
                    contiguous = False
                rows.append((g.data_ptr(), self.layout.offsets[i], p.numel(), local[gi], i))
            key = tuple(rows)
            hit = self._segment_tables.get(key)
            if hit is None:
                table, nchunks = segment_table(rows, CHUNK)
                if len(self._segment_tables) >= 4:
                    self._segment_tables.clear()
                hit = self._segment_tables[key] = (upload(table, self.device), len(rows), nchunks)
            self._segments, self._num_segments, self._num_chunks = hit
            # Non-contiguous gradients are copied every step: nothing to reuse then.
            self._rows_cache = (fast_key, entries) if contiguous else None
        group_array = (N.AdamWGroup * len(structs))(*structs)
        args = N.AdamWMtArgs(
            param=self.master.data_ptr(), exp_avg=self.exp_avg.data_ptr(), exp_avg_sq=self.exp_avg_sq.data_ptr(),
            model_copy=None if self.copy is None else self.copy.data_ptr(),
            model_dtype=0 if self.copy is None else N.dtype_code(self.model_dtype),
            grad_dtype=N.dtype_code(self.grad_dtype), segments=self._segments.data_ptr(),
            num_segments=self._num_segments, chunk_elems=CHUNK, num_chunks=self._num_chunks,
            steps=self.steps.data_ptr(), corrections=self.corrections.tensor.data_ptr(),
            correction_capacity=self.corrections.capacity,
            scale=None if scale is None else scale.data_ptr(), stats=None if stats is None else stats.data_ptr(),
            skip_nonfinite=int(skip_nonfinite), clip=int(max_norm is not None),
            max_norm=float(max_norm) if max_norm is not None else 0.0,
            workspace=self.workspace.data_ptr(), error=self.error.data_ptr(),
            groups=group_array, num_groups=len(structs))
        if schedule is not None:
            args.lr_schedule, args.lr_schedule_rows, args.lr_schedule_columns, args.lr_step = schedule
        N.call("nt_adamw_mt", N.C.byref(args), N.stream_handle())
        del keep

    # ---- state export / import --------------------------------------------------------------
    def has_state(self, steps: list[int], i: int) -> bool:
        return steps[i] > 0 or i in self.loaded

    def export(self) -> list[dict | None]:
        steps = self.steps.cpu().tolist()
        out: list[dict | None] = []
        for i in range(len(self.params)):
            if not self.has_state(steps, i):
                out.append(None)
                continue
            entry = {"step": int(steps[i]),
                     "exp_avg": self.view(self.exp_avg, i).detach().clone(),
                     "exp_avg_sq": self.view(self.exp_avg_sq, i).detach().clone()}
            if self.copy is not None:
                entry["master_param"] = self.master_view(i).detach().clone()
            out.append(entry)
        return out

    def load(self, states: dict[int, dict]) -> None:
        """Installs per-parameter state; parameters absent from ``states`` restart from zero."""
        self.ensure_moments()
        steps = [0] * len(self.params)
        self.loaded = set()
        with torch.no_grad():
            for i in range(len(self.params)):
                st = states.get(i)
                if not st:
                    self.view(self.exp_avg, i).zero_()
                    self.view(self.exp_avg_sq, i).zero_()
                    continue
                self.view(self.exp_avg, i).copy_(st["exp_avg"])
                self.view(self.exp_avg_sq, i).copy_(st["exp_avg_sq"])
                if "master_param" in st:
                    self.master_view(i).copy_(st["master_param"])
                    if self.copy is not None:
                        self.view(self.copy, i).copy_(self.master_view(i).to(self.model_dtype))
                steps[i] = int(st["step"])
                self.loaded.add(i)
            self.steps.copy_(torch.tensor(steps, dtype=torch.int32))
        self.max_step = max(steps) if steps else 0
        self._segment_tables.clear()
