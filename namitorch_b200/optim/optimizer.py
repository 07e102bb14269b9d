"""Optimizer base: parameter groups, gradient discovery, zero_grad and the state-dict format.

Mirrors namitorch/optim/optimizer.py:96-315 (messages, validation order, version-1
state_dict with parameters referenced by index) for torch CUDA tensors standing in for
the reference's Parameter objects.
"""
from __future__ import annotations

import copy

import torch


def _parameter_list(params, path: str, allow_single: bool = False) -> list[torch.Tensor]:
    """namitorch/optim/optimizer.py:96-117."""
    if allow_single and isinstance(params, torch.Tensor):
        values = [params]
    else:
        if isinstance(params, (torch.Tensor, dict, str, bytes, set, frozenset)):
            raise TypeError(f"{path} must be an ordered iterable of Parameters.")
        try:
            values = list(params)
        except TypeError:
            raise TypeError(f"{path} must be an ordered iterable of Parameters.") from None
    if not values:
        raise ValueError(f"{path} cannot be empty.")
    identities = set()
    for parameter in values:
        if not isinstance(parameter, torch.Tensor):
            raise TypeError(f"{path} must contain only NamiTorch Parameters, got {type(parameter).__name__}.")
        if not parameter.is_leaf:
            raise ValueError(f"{path} must contain only leaf Parameters.")
        if id(parameter) in identities:
            raise ValueError(f"{path} contains a duplicate Parameter object.")
        identities.add(id(parameter))
    return values


def _copy_options(options: dict, path: str) -> dict:
    """namitorch/optim/optimizer.py:86-93."""
    if not isinstance(options, dict):
        raise TypeError(f"{path} must be a dictionary.")
    if any(not isinstance(key, str) or not key for key in options):
        raise TypeError(f"{path} option names must be nonempty strings.")
    if "params" in options:
        raise ValueError(f"{path} cannot contain the reserved option 'params'.")
    return copy.deepcopy(options)


class Optimizer:
    def __init__(self, params, defaults: dict | None = None):
        self.defaults = self._prepare_options({} if defaults is None else defaults, "defaults")
        self.param_groups: list[dict] = []
        if isinstance(params, (torch.Tensor, dict, str, bytes, set, frozenset)):
            raise TypeError("Optimizer params must be an ordered iterable of Parameters or parameter-group dictionaries.")
        try:
            entries = list(params)
        except TypeError:
            raise TypeError("Optimizer params must be an ordered iterable of Parameters or parameter-group dictionaries.") from None
        if not entries:
            raise ValueError("Optimizer cannot receive an empty parameter list.")
        if all(isinstance(entry, dict) for entry in entries):
            groups = entries
        elif any(isinstance(entry, dict) for entry in entries):
            raise TypeError("Optimizer params cannot mix Parameters and parameter-group dictionaries.")
        else:
            groups = [{"params": entries}]
        for group in groups:
            self.add_param_group(group)

    def _prepare_options(self, options: dict, path: str) -> dict:
        return _copy_options(options, path)

    def _group_signature(self):
        """Identity of the group structure and of every registered parameter (cheap)."""
        try:
            return tuple((id(group), id(group["params"]), tuple(map(id, group["params"])))
                         for group in self.param_groups)
        except Exception:   # malformed groups: the full validation below reports them
            return None

    def _registered_parameters(self) -> list[torch.Tensor]:
        """namitorch/optim/optimizer.py:148-164. The validated list is kept until the groups or
        their parameter objects change (an identity check of every entry per call)."""
        signature = self._group_signature()
        cached = self.__dict__.get("_registered_cache")
        if signature is not None and cached is not None and cached[0] == signature:
            return cached[1]
        parameters = self._validate_registered()
        if signature is not None:
            self._registered_cache = (signature, parameters)
        return parameters

    def _validate_registered(self) -> list[torch.Tensor]:
        if not self.param_groups:
            raise ValueError("Optimizer must contain at least one parameter group.")
        parameters = []
        identities = set()
        for index, group in enumerate(self.param_groups):
            if not isinstance(group, dict) or "params" not in group:
                raise TypeError(f"Parameter group {index} must be a dictionary containing 'params'.")
            if not isinstance(group["params"], list):
                raise TypeError(f"Parameter group {index} params must remain a materialized list.")
            current = _parameter_list(group["params"], f"param_groups[{index}]['params']")
            for parameter in current:
                if id(parameter) in identities:
                    raise ValueError("A Parameter object cannot belong to more than one parameter group.")
                identities.add(id(parameter))
            parameters.extend(current)
        return parameters

    def add_param_group(self, param_group: dict) -> None:
        """namitorch/optim/optimizer.py:166-179."""
        if not isinstance(param_group, dict):
            raise TypeError("add_param_group requires a dictionary.")
        if "params" not in param_group:
            raise ValueError("A parameter group must contain 'params'.")
        parameters = _parameter_list(param_group["params"], "param_group['params']", allow_single=True)
        existing = {id(parameter) for parameter in self._registered_parameters()} if self.param_groups else set()
        if any(id(parameter) in existing for parameter in parameters):
            raise ValueError("A Parameter object cannot belong to more than one parameter group.")
        options = _copy_options(self.defaults, "defaults")
        options.update(_copy_options({key: value for key, value in param_group.items() if key != "params"},
                                     "param_group"))
        options = self._prepare_options(options, "param_group")
        options["params"] = parameters
        self.param_groups.append(options)
        self._on_param_group_added()

    def _on_param_group_added(self) -> None:
        pass

    def _parameters_with_grad(self):
        """namitorch/optim/optimizer.py:181-195."""
        for _, group, parameter, gradient in self._grad_entries():
            yield group, parameter, gradient

    def _grad_entries(self) -> list:
        """[(group index, group, parameter, gradient)] of the parameters that have gradients,
        validated as the reference does. The list is kept while the same gradient objects sit
        on the same parameters (checked by identity every call); a new gradient object is
        validated again."""
        parameters = self._registered_parameters()
        gradients = [parameter.grad for parameter in parameters]
        key = (id(parameters), tuple(map(id, gradients)), tuple(parameter.requires_grad for parameter in parameters))
        cached = self.__dict__.get("_entries_cache")
        if cached is not None and cached[0] == key:
            return cached[1]
        entries = []
        for index, group in enumerate(self.param_groups):
            for parameter in group["params"]:
                if not parameter.requires_grad or parameter.grad is None:
                    continue
                gradient = parameter.grad
                if not isinstance(gradient, torch.Tensor):
                    raise TypeError("Parameter gradients must be NamiTorch Tensors.")
                if gradient.device != parameter.device:
                    raise RuntimeError(f"Operands are on different devices: {parameter.device}, {gradient.device}; "
                                       "use an explicit .to() transfer.")
                if gradient.shape != parameter.shape:
                    raise ValueError(f"Gradient shape {tuple(gradient.shape)} does not match parameter shape "
                                     f"{tuple(parameter.shape)}.")
                if gradient.dtype is not parameter.dtype:
                    raise TypeError(f"Gradient dtype {gradient.dtype} does not match parameter dtype {parameter.dtype}.")
                entries.append((index, group, parameter, gradient))
        # The gradients list keeps the objects alive, so their ids stay unique while cached.
        self._entries_cache = (key, entries, gradients)
        return entries

    def zero_grad(self, set_to_none: bool = True) -> None:
        """namitorch/optim/optimizer.py:197-206."""
        if type(set_to_none) is not bool:
            raise TypeError("set_to_none must be a Python bool.")
        parameters = self._registered_parameters()
        with torch.no_grad():
            for parameter in parameters:
                if set_to_none:
                    parameter.grad = None
                elif parameter.grad is not None:
                    parameter.grad.zero_()

    def step(self, closure=None):
        raise RuntimeError("Optimizer subclass must implement step.")

    # ---- state dict (format of namitorch/optim/optimizer.py:211-233) ----------------------
    def _export_state(self, parameters: list[torch.Tensor]) -> dict[int, dict]:
        return {}

    def _import_state(self, index_to_parameter: dict[int, torch.Tensor], saved_state: dict) -> None:
        pass

    def state_dict(self) -> dict:
        parameters = self._registered_parameters()
        indices = {id(parameter): index for index, parameter in enumerate(parameters)}
        groups = []
        for index, group in enumerate(self.param_groups):
            copied = self._prepare_options({key: value for key, value in group.items() if key != "params"},
                                           f"param_groups[{index}]")
            copied["params"] = [indices[id(parameter)] for parameter in group["params"]]
            groups.append(copied)
        return {
            "version": 1,
            "defaults": self._prepare_options(self.defaults, "defaults"),
            "param_groups": groups,
            "param_shapes": [list(parameter.shape) for parameter in parameters],
            # Per-parameter fields in sorted order, as the reference's state copy emits them
            # (so a checkpoint archive of this state has the reference's metadata bytes).
            "state": {index: {name: values[name] for name in sorted(values)}
                      for index, values in self._export_state(parameters).items()},
        }

    def load_state_dict(self, state_dict: dict) -> None:
        """Validation of namitorch/optim/optimizer.py:235-286, then the state is installed."""
        if not isinstance(state_dict, dict):
            raise TypeError("Optimizer state_dict must be a dictionary.")
        expected_keys = {"version", "defaults", "param_groups", "param_shapes", "state"}
        if set(state_dict) != expected_keys:
            raise ValueError("Optimizer state_dict must contain version, defaults, param_groups, param_shapes and state.")
        if type(state_dict["version"]) is not int or state_dict["version"] != 1:
            raise ValueError("Unsupported optimizer state_dict version.")
        parameters = self._registered_parameters()
        groups = state_dict["param_groups"]
        if not isinstance(groups, list) or len(groups) != len(self.param_groups):
            raise ValueError("Loaded optimizer must have the same number of parameter groups.")
        shapes = state_dict["param_shapes"]
        if not isinstance(shapes, list) or len(shapes) != len(parameters):
            raise ValueError("Loaded optimizer must contain one shape for each parameter.")
        defaults = self._prepare_options(state_dict["defaults"], "defaults")
        restored_groups = []
        index_to_parameter = {}
        for group_index, (saved, current) in enumerate(zip(groups, self.param_groups)):
            if not isinstance(saved, dict) or "params" not in saved:
                raise ValueError(f"Loaded parameter group {group_index} must contain 'params'.")
            saved_indices = saved["params"]
            if not isinstance(saved_indices, list) or len(saved_indices) != len(current["params"]):
                raise ValueError(f"Loaded parameter group {group_index} has a different number of parameters.")
            options = self._prepare_options({key: value for key, value in saved.items() if key != "params"},
                                            f"param_groups[{group_index}]")
            if not defaults.keys() <= options.keys():
                raise ValueError(f"Loaded parameter group {group_index} is missing default options.")
            for index, parameter in zip(saved_indices, current["params"]):
                if type(index) is not int or not 0 <= index < len(parameters):
                    raise ValueError("Loaded parameter indices must be integers in the registered parameter range.")
                if index in index_to_parameter:
                    raise ValueError("Loaded parameter groups contain duplicate parameter indices.")
                shape = shapes[index]
                if not isinstance(shape, (list, tuple)) or any(type(d) is not int or d < 0 for d in shape):
                    raise ValueError(f"Invalid saved parameter shape for index {index}.")
                if tuple(shape) != tuple(parameter.shape):
                    raise ValueError(f"Saved parameter {index} shape {tuple(shape)} does not match current shape "
                                     f"{tuple(parameter.shape)}.")
                index_to_parameter[index] = parameter
            options["params"] = list(current["params"])
            restored_groups.append(options)
        saved_state = state_dict["state"]
        if not isinstance(saved_state, dict):
            raise TypeError("Loaded optimizer state must be a dictionary keyed by parameter indices.")
        for index, values in saved_state.items():
            if type(index) is not int or index not in index_to_parameter:
                raise ValueError("Loaded state keys must be registered parameter indices.")
            if not isinstance(values, dict):
                raise TypeError(f"Loaded state[{index}] must be a dictionary.")
        # The loaded groups decide where the state lives (their `fused` option selects the
        # multi-tensor arenas or per-tensor buffers), so they are installed first and put
        # back if the state is rejected.
        previous = (self.defaults, self.param_groups)
        self.defaults, self.param_groups = defaults, restored_groups
        try:
            self._import_state(index_to_parameter, saved_state)
        except BaseException:
            self.defaults, self.param_groups = previous
            raise

    def __repr__(self) -> str:
        return f"{type(self).__name__}(param_groups={len(self.param_groups)})"
