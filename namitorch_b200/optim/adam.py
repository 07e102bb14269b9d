"""Adam and AdamW with the reference's API (namitorch/optim/adam.py:8-97).

``AdamW(params, lr, betas, eps, weight_decay, *, maximize, fused)`` keeps the reference
signature. On the CUDA path every parameter lives in flat arenas (see ``_engine``) and one
multi-tensor kernel launch updates all of them; ``fused=False`` (or
``enable_fused_kernels(False)`` with ``fused=None``) instead launches the per-tensor kernel
once per parameter through the ``backend.adamw`` seam, the reference's launch pattern
(namitorch/optim/adam.py:69-94). Both run the same float32 operation sequence and agree
bit for bit with the reference NumPy path. There is no CPU fallback.

Extension: ``model_dtype=torch.bfloat16`` (or float16) keeps fp32 master weights inside the
optimizer and turns the parameters into views of a low-precision model copy that the
update kernel rewrites in the same pass; gradients then arrive in that dtype.
"""
from __future__ import annotations

import weakref

import numpy as np
import torch

from .. import _native as N
from ..backends import fused_kernels_enabled
from ..backends.cuda import AdamWCUDAKernel
from ..flat import grad_stats_for, launch_transform, stats_tensor
from ._common import _bool_option, _real_option, _scalar
from ._engine import FusedAdamEngine
from .optimizer import Optimizer

# id(parameter) -> optimizer whose engine owns it (used by clip_grad_norm_ to defer clipping).
_OWNERS: "weakref.WeakValueDictionary[int, _FirstOrderAdam]" = weakref.WeakValueDictionary()


def _owner_of(parameter: torch.Tensor):
    return _OWNERS.get(id(parameter))


class _AmpPending:
    """Unscale / clip factors that the next fused step applies instead of rewriting gradients."""

    def __init__(self, key, stats, scale):
        self.key = key            # identity of the gradients the statistics were taken over
        self.stats = stats        # device nt_stats (found_inf, norm)
        self.scale = scale        # device loss scale still to divide by, or None
        self.skip = False         # skip the step when stats.found_inf (set by GradScaler)
        self.max_norm = None      # pending clip_grad_norm_ bound, or None


class _StateView:
    """``optimizer.state`` keyed by ``id(parameter)``; reading it synchronises with the device."""

    def __init__(self, optimizer):
        self._opt = optimizer

    def _table(self) -> dict[int, dict]:
        return self._opt._state_by_id()

    def __getitem__(self, key):
        return self._table().get(key, {})

    def get(self, key, default=None):
        return self._table().get(key, default)

    def __contains__(self, key):
        return key in self._table()

    def __iter__(self):
        return iter(self._table())

    def __len__(self):
        return len(self._table())

    def items(self):
        return self._table().items()

    def keys(self):
        return self._table().keys()

    def values(self):
        return self._table().values()


class _FirstOrderAdam(Optimizer):
    _decoupled_weight_decay = False

    def __init__(self, params, defaults: dict, model_dtype=None):
        self._engine: FusedAdamEngine | None = None
        self._model_dtype = model_dtype
        self._per_tensor_state: dict[int, dict] = {}
        self._amp: _AmpPending | None = None
        super().__init__(params, defaults)
        self.state = _StateView(self)
        # The arenas are built now, not at the first step: the parameters must already be
        # views of the model copy (in its dtype) when the first gradients are assigned.
        if self._uses_engine():
            self._ensure_engine()

    # ---- options (namitorch/optim/_common.py:83-88, adam.py:17-25, :52-56) -------------------
    def _prepare_options(self, options: dict, path: str) -> dict:
        prepared = super()._prepare_options(options, path)
        if path == "defaults" and not options:
            return prepared
        _real_option(prepared, "lr")
        _real_option(prepared, "weight_decay")
        _bool_option(prepared, "maximize")
        _real_option(prepared, "eps", positive=True)
        betas = prepared.get("betas")
        if not isinstance(betas, (tuple, list)) or len(betas) != 2:
            raise TypeError("Adam betas must contain exactly two real scalars.")
        normalized = {"beta1": betas[0], "beta2": betas[1]}
        prepared["betas"] = tuple(_real_option(normalized, name, unit_interval=True) for name in ("beta1", "beta2"))
        return prepared

    def _uses_engine(self) -> bool:
        return True

    def _on_param_group_added(self) -> None:
        if self._engine is not None:
            raise RuntimeError("add_param_group after the flat arenas were built is not supported; "
                               "create the optimizer with every parameter group.")

    def _ensure_engine(self) -> FusedAdamEngine:
        if self._engine is None:
            params = self._registered_parameters()
            self._engine = FusedAdamEngine(params, model_dtype=self._model_dtype)
            for p in params:
                _OWNERS[id(p)] = self
        return self._engine

    def _entries(self):
        """[(group index, parameter, gradient)], the same list object while nothing changed."""
        full = self._grad_entries()
        cached = self.__dict__.get("_entries_view")
        if cached is not None and cached[0] is full:
            return cached[1]
        view = [(index, parameter, gradient) for index, _, parameter, gradient in full]
        self._entries_view = (full, view)
        return view

    def _validated_options(self) -> list[dict]:
        options = [self._prepare_options({k: v for k, v in group.items() if k != "params"}, "param_group")
                   for group in self.param_groups]
        for prepared in options:
            for name, value in prepared.items():
                if type(value) is float:
                    _scalar(value, name)
            if self._decoupled_weight_decay:
                _scalar(1 - prepared["lr"] * prepared["weight_decay"], "decay factor")
        return options

    # ---- step -------------------------------------------------------------------------------
    def step(self, closure=None):
        """namitorch/optim/_common.py:133-167, with every parameter updated by one launch."""
        if torch.cuda.is_available() and torch.cuda.is_current_stream_capturing():
            from ..training import capture_in_progress
            if not capture_in_progress():
                raise RuntimeError("Optimizer steps are not allowed during CUDA graph capture (use "
                                   "namitorch_b200.training.CapturedOptimizerStep).")
        if closure is not None and not callable(closure):
            raise TypeError("Optimizer closure must be callable or None.")
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()
        options = self._validated_options()
        if self._uses_engine():
            engine = self._ensure_engine()
            entries = self._entries()
            amp = self._amp
            self._amp = None
            if amp is not None and amp.key != self._grad_key(entries):
                raise RuntimeError("Optimizer gradients changed after unscale_; clipping must modify the existing "
                                   "gradients in-place.")
            engine.step(entries, options, decoupled=self._decoupled_weight_decay,
                        scale=None if amp is None else amp.scale, stats=None if amp is None else amp.stats,
                        skip_nonfinite=bool(amp is not None and amp.skip),
                        max_norm=None if amp is None else amp.max_norm, schedule=self._device_schedule())
        else:
            if self._device_schedule() is not None:
                raise RuntimeError("A device-gated learning-rate schedule needs the fused multi-tensor path "
                                   "(fused=None or True).")
            self._per_tensor_step(options)
        return loss

    def _device_schedule(self):
        """(table, rows, columns, step) of a scheduler that moved its step to the device."""
        scheduler = getattr(self, "_lr_schedule", None)
        return None if scheduler is None else scheduler._schedule_args()

    def _per_tensor_step(self, options):
        raise NotImplementedError

    # ---- AMP / clipping hooks used by GradScaler and clip_grad_norm_ ------------------------
    def _grad_key(self, entries) -> tuple:
        """Identity and storage of every gradient (the GradScaler checks that clipping kept them)."""
        return (tuple(id(p) for _, p, _ in entries),
                tuple(map(id, (g for _, _, g in entries))),
                tuple(map(torch.Tensor.data_ptr, (g for _, _, g in entries))))

    def _amp_gradients(self) -> list[torch.Tensor]:
        return [g for _, _, g in self._entries()]

    def _amp_unscale_(self, scale: torch.Tensor, lazy: bool) -> torch.Tensor:
        """Statistics of the unscaled gradients; ``lazy`` defers the division to the update."""
        entries = self._entries()
        grads = [g for _, _, g in entries]
        if self._uses_engine():
            self._ensure_engine()
        if lazy and self._uses_engine():
            stats = grad_stats_for(grads, scale=scale)
            self._amp = _AmpPending(self._grad_key(entries), stats, scale)
        else:
            launch_transform(grads, scale=scale)
            stats = grad_stats_for(grads)
            self._amp = _AmpPending(self._grad_key(entries), stats, None)
        return stats

    def _amp_enable_skip(self) -> None:
        if self._amp is not None:
            self._amp.skip = True

    def _lazy_clip(self, max_norm: float, norm_type: float, check=None) -> torch.Tensor | None:
        """Defers clip_grad_norm_ to the update when it covers exactly this optimizer's gradients.

        ``check(stats)`` runs before anything is registered, so an error_if_nonfinite failure
        leaves no pending clip behind."""
        if not self._uses_engine():
            return None
        entries = self._entries()
        key = self._grad_key(entries)
        amp = self._amp
        if amp is not None and (amp.key != key or amp.max_norm is not None):
            return None
        if amp is not None and norm_type == 2.0:
            stats = amp.stats
        else:
            grads = [g for _, _, g in entries]
            stats = grad_stats_for(grads, scale=None if amp is None else amp.scale, norm_type=norm_type)
            if amp is not None:
                # found_inf for the skip stays with the unscale statistics; the norm comes from these.
                merged = amp.stats.clone()
                merged[N.STATS_FIELDS.index("norm")] = stats[N.STATS_FIELDS.index("norm")]
                stats = merged
        if check is not None:
            check(stats)
        if amp is None:
            amp = _AmpPending(key, stats, None)
        else:
            amp.stats = stats
        amp.max_norm = float(max_norm)
        self._amp = amp
        return stats

    def _materialize_pending(self) -> None:
        """Writes deferred unscale / clip factors into the gradient storage."""
        amp = self._amp
        if amp is None or (amp.scale is None and amp.max_norm is None):
            return
        grads = self._amp_gradients()
        launch_transform(grads, scale=amp.scale, stats=amp.stats, max_norm=amp.max_norm)
        amp.scale = None
        amp.max_norm = None

    # ---- state ------------------------------------------------------------------------------
    def _state_by_id(self) -> dict[int, dict]:
        if not self._uses_engine():
            return dict(self._per_tensor_state)
        if self._engine is None:
            return {}
        exported = self._engine.export()
        table = {}
        for i, p in enumerate(self._engine.params):
            if exported[i] is None:
                continue
            entry = dict(exported[i])
            entry["exp_avg"] = self._engine.view(self._engine.exp_avg, i)
            entry["exp_avg_sq"] = self._engine.view(self._engine.exp_avg_sq, i)
            table[id(p)] = entry
        return table

    def _allowed_state_fields(self) -> set[str]:
        allowed = {"step", "exp_avg", "exp_avg_sq"}
        if self._model_dtype is not None:
            allowed.add("master_param")
        return allowed

    def _export_state(self, parameters) -> dict[int, dict]:
        indices = {id(p): k for k, p in enumerate(parameters)}
        if not self._uses_engine():
            return {indices[pid]: {"step": st["step"], "exp_avg": st["exp_avg"].clone(),
                                   "exp_avg_sq": st["exp_avg_sq"].clone()}
                    for pid, st in self._per_tensor_state.items()}
        if self._engine is None:
            return {}
        exported = self._engine.export()
        return {indices[id(p)]: exported[i] for i, p in enumerate(self._engine.params) if exported[i] is not None}

    def _check_state(self, values: dict, parameter: torch.Tensor, path: str) -> None:
        """namitorch/optim/_common.py:98-130 for state being loaded."""
        if not isinstance(values, dict):
            raise TypeError(f"{path} must be a dictionary.")
        if not values:
            return
        allowed = self._allowed_state_fields()
        required = {"step", "exp_avg", "exp_avg_sq"}
        if not set(values) <= allowed or not required <= values.keys():
            raise ValueError(f"{path} has invalid state fields for {type(self).__name__}.")
        if type(values["step"]) is not int or values["step"] < 0:
            raise ValueError(f"{path} step must be a nonnegative Python integer.")
        for name in sorted(set(values) - {"step"}):
            value = values[name]
            if isinstance(value, np.ndarray):
                value = torch.from_numpy(value)
            if not isinstance(value, torch.Tensor):
                raise TypeError(f"{path}[{name!r}] must be a floating Tensor or NumPy array.")
            if not value.dtype.is_floating_point:
                raise TypeError(f"{path}[{name!r}] must have a floating dtype.")
            if tuple(value.shape) != tuple(parameter.shape):
                raise ValueError(f"{path}[{name!r}] shape {tuple(value.shape)} must equal parameter shape "
                                 f"{tuple(parameter.shape)}.")
            if name == "exp_avg_sq" and bool((value < 0).any()):
                raise ValueError(f"{path}[{name!r}] must be nonnegative.")

    def _import_state(self, index_to_parameter, saved_state) -> None:
        by_param = {}
        for index, values in saved_state.items():
            parameter = index_to_parameter[index]
            self._check_state(values, parameter, f"state[{index}]")
            if not values:
                continue
            converted = {"step": values["step"]}
            for name in set(values) - {"step"}:
                v = values[name]
                v = torch.from_numpy(v) if isinstance(v, np.ndarray) else v
                converted[name] = v.detach().to(device=parameter.device, dtype=torch.float32)
            by_param[id(parameter)] = converted
        if self._uses_engine():
            engine = self._ensure_engine()
            engine.load({engine.index[pid]: st for pid, st in by_param.items()})
        else:
            self._per_tensor_state = {pid: {"step": st["step"], "exp_avg": st["exp_avg"].clone(),
                                            "exp_avg_sq": st["exp_avg_sq"].clone()} for pid, st in by_param.items()}

    def to(self, device):
        """Optimizer state already lives beside the parameters; moving it elsewhere is rejected
        the way the reference rejects a move ahead of the parameters (optimizer.py:288-309)."""
        target = torch.device(device)
        for p in self._registered_parameters():
            if p.device != target and not (target.index is None and p.device.type == target.type):
                raise RuntimeError(f"Move all optimizer parameters to {target} first with model.to(device); "
                                   "optimizer.to(device) moves only optimizer state.")
        return self

    @property
    def master_params(self) -> list[torch.Tensor]:
        """fp32 master weights (views), in registration order."""
        engine = self._ensure_engine()
        return [engine.master_view(i) for i in range(len(engine.params))]


class Adam(_FirstOrderAdam):
    """namitorch/optim/adam.py:8-42: L2 weight decay added to the gradient."""

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 0.0,
                 *, maximize: bool = False, model_dtype=None):
        super().__init__(params, {"lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay,
                                  "maximize": maximize}, model_dtype=model_dtype)


class AdamW(_FirstOrderAdam):
    """namitorch/optim/adam.py:45-94: decoupled weight decay, ``fused`` switch."""

    _decoupled_weight_decay = True

    def __init__(self, params, lr: float = 1e-3, betas=(0.9, 0.999), eps: float = 1e-8, weight_decay: float = 1e-2,
                 *, maximize: bool = False, fused=None, model_dtype=None):
        if fused is False and model_dtype is not None:
            raise ValueError("model_dtype requires the multi-tensor path (fused=None or True).")
        super().__init__(params, {"lr": lr, "betas": betas, "eps": eps, "weight_decay": weight_decay,
                                  "maximize": maximize, "fused": fused}, model_dtype=model_dtype)

    def _prepare_options(self, options: dict, path: str) -> dict:
        prepared = super()._prepare_options(options, path)
        fused = prepared.setdefault("fused", None)
        if fused is not None and type(fused) is not bool:
            raise TypeError("AdamW fused must be None, True or False.")
        return prepared

    def _uses_engine(self) -> bool:
        modes = {group.get("fused", None) for group in self.param_groups}
        if modes == {False} or (modes <= {None, False} and not fused_kernels_enabled() and self._engine is None):
            if self._model_dtype is not None:
                raise RuntimeError("model_dtype requires the multi-tensor path (fused=None or True).")
            return False
        if False in modes:
            raise RuntimeError("AdamW groups must agree on fused=False versus the multi-tensor path.")
        return True

    def _per_tensor_step(self, options):
        """One launch per parameter through the backend.adamw seam (namitorch/optim/adam.py:69-94)."""
        kernel = AdamWCUDAKernel()
        amp = self._amp
        self._amp = None
        if amp is not None and amp.skip and bool(amp.stats[N.STATS_FIELDS.index("found_inf")].item() != 0):
            return
        for gi, parameter, gradient in self._entries():
            o = options[gi]
            state = self._per_tensor_state.get(id(parameter)) or {}
            if "exp_avg" not in state:
                state["exp_avg"] = torch.zeros_like(parameter)
                state["exp_avg_sq"] = torch.zeros_like(parameter)
            if not kernel.supports(parameter, gradient, state["exp_avg"], state["exp_avg_sq"]):
                raise RuntimeError("fused=True requires non-overlapping contiguous float32 CUDA parameters, "
                                   "gradients and states on the same device.")
            step = state.get("step", 0) + 1
            beta1, beta2 = o["betas"]
            coefficients = tuple(_scalar(value) for value in (
                o["lr"], beta1, beta2, 1 - beta1, 1 - beta2, o["eps"], o["weight_decay"],
                1 - o["lr"] * o["weight_decay"], 1 - beta1 ** step, 1 - beta2 ** step))
            kernel.run(parameter, gradient, state["exp_avg"], state["exp_avg_sq"], coefficients=coefficients,
                       maximize=o["maximize"], update_parameter=o["lr"] != 0)
            state["step"] = step
            self._per_tensor_state[id(parameter)] = state


__all__ = ["Adam", "AdamW"]
