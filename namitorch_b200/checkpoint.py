"""Checkpoint archives in the reference's on-disk format.

The reference stores an object tree as one uncompressed zip archive
(namitorch/serialization.py:75-107, read back by :192-253): ``metadata.json`` holds
``{"format_version": 1, "tree": ..., "arrays": [...]}``, where the tree tags every node
with its type (none / bool / int / str / float as a hex string / list / tuple / dict with
string keys / tensor / ndarray) and every array node refers by id (``a0``, ``a1``, ...) to
an NPY 1.0 entry ``<id>.npy`` of the nested uncompressed zip ``arrays.npz``. This module
reads and writes that format with the reference's validation rules, and packs optimizers
the way namitorch/training/checkpoint.py:59-77 does (state indices as decimal strings), so
optimizer and GradScaler state move between the reference and this package in both
directions. Writing the same tree gives the same ``metadata.json`` bytes.

Tensor nodes decode to CPU torch tensors (``requires_grad`` kept), ndarray nodes to NumPy
arrays. The format's array dtypes are NumPy's bool, int8-64, uint8-64 and float16/32/64:
a bfloat16 tensor is rejected (store it as float32).
"""
from __future__ import annotations

import json
import math
import os
import tempfile
import zipfile
from contextlib import contextmanager
from numbers import Integral
from pathlib import Path

import numpy as np
import torch

FORMAT_VERSION = 1
CHECKPOINT_VERSION = 1
_MAX_DEPTH = 128
_MAX_METADATA_BYTES = 16 * 1024 * 1024
_ARRAY_KINDS = {"b": (1,), "i": (1, 2, 4, 8), "u": (1, 2, 4, 8), "f": (2, 4, 8)}
_CHECKPOINT_KEYS = {"checkpoint_version", "model", "optimizer", "optimizer_type", "optimizer_parameter_names",
                    "scheduler", "rng", "step", "epoch", "config", "cumulative_tokens"}


class SerializationError(ValueError):
    """An archive that does not follow the format (same class role as the reference's)."""
    __slots__ = ()


def _checked_dtype(text) -> np.dtype:
    if not isinstance(text, str):
        raise SerializationError("Array dtype must be a string.")
    dtype = np.dtype(text)
    if (dtype.kind not in _ARRAY_KINDS or dtype.itemsize not in _ARRAY_KINDS[dtype.kind] or dtype.fields is not None
            or dtype.subdtype is not None):
        raise SerializationError(f"Unsupported archive array dtype {text!r}; object and complex arrays are forbidden.")
    if dtype.str != text:
        raise SerializationError("Array dtype must use its canonical NumPy dtype string.")
    return dtype


# ---- writing ---------------------------------------------------------------------------------
def _array_of(value) -> tuple[np.ndarray, dict]:
    if isinstance(value, torch.Tensor):
        if value.dtype == torch.bfloat16:
            raise SerializationError("bfloat16 has no NumPy dtype in the archive format; convert it to float32.")
        array = value.detach().to("cpu").numpy()
        return array, {"type": "tensor", "requires_grad": bool(value.requires_grad)}
    return value, {"type": "ndarray"}


def _to_tree(value, arrays: list, active: set, depth: int = 0):
    if depth > _MAX_DEPTH:
        raise SerializationError(f"Archive nesting exceeds {_MAX_DEPTH} levels.")
    if value is None:
        return {"type": "none"}
    if type(value) in (bool, int, str):
        return {"type": type(value).__name__, "value": value}
    if type(value) is float:
        return {"type": "float", "value": value.hex()}
    if isinstance(value, (torch.Tensor, np.ndarray)):
        array, head = _array_of(value)
        if array.dtype.metadata is not None:
            raise SerializationError("Array dtypes with custom metadata are unsupported.")
        _checked_dtype(array.dtype.str)
        ident = f"a{len(arrays)}"
        arrays.append((ident, array))
        node = {"type": head["type"], "id": ident}
        if head["type"] == "tensor":
            node["requires_grad"] = head["requires_grad"]
        return node
    if not isinstance(value, (list, tuple, dict)):
        raise TypeError(f"Cannot serialize {type(value).__name__}; only primitive containers, Tensor and ndarray "
                        "are supported.")
    if id(value) in active:
        raise SerializationError("Cannot serialize cyclic containers.")
    active.add(id(value))
    try:
        if isinstance(value, dict):
            if any(type(key) is not str for key in value):
                raise TypeError("Archive dictionaries require string keys.")
            return {"type": "dict", "items": [[key, _to_tree(item, arrays, active, depth + 1)]
                                              for key, item in value.items()]}
        return {"type": "tuple" if isinstance(value, tuple) else "list",
                "items": [_to_tree(item, arrays, active, depth + 1) for item in value]}
    finally:
        active.discard(id(value))


def metadata_bytes(obj) -> tuple[bytes, list]:
    """(the archive's metadata.json bytes, [(id, array)]) for `obj`."""
    arrays: list = []
    tree = _to_tree(obj, arrays, set())
    metadata = {"format_version": FORMAT_VERSION, "tree": tree,
                "arrays": [{"id": ident, "dtype": a.dtype.str, "shape": list(a.shape), "nbytes": int(a.nbytes)}
                           for ident, a in arrays]}
    encoded = json.dumps(metadata, ensure_ascii=True, allow_nan=False, separators=(",", ":")).encode("utf-8")
    if len(encoded) > _MAX_METADATA_BYTES:
        raise SerializationError("Archive metadata exceeds the 16 MiB format limit.")
    return encoded, arrays


@contextmanager
def _replacing(target: Path):
    """A temporary file beside `target`, open for writing. When the block ends normally it is
    flushed to disk and renamed over `target` (readers see the old or the new archive, never
    a partial one); when it raises, the temporary file is removed."""
    handle, name = tempfile.mkstemp(dir=target.parent, prefix=f".{target.name}.", suffix=".tmp")
    staged = Path(name)
    try:
        with os.fdopen(handle, "w+b") as out:
            yield out
            out.flush()
            os.fsync(out.fileno())
        os.replace(staged, target)
    except BaseException:
        staged.unlink(missing_ok=True)
        raise


def _stored_zip(handle) -> zipfile.ZipFile:
    """A ZIP writer without compression (the format stores every member as is)."""
    return zipfile.ZipFile(handle, "w", compression=zipfile.ZIP_STORED, allowZip64=True)


def _write_arrays(npz: zipfile.ZipFile, arrays) -> None:
    """One NPY 1.0 member per array, from a C-ordered snapshot taken as it is written."""
    for ident, array in arrays:
        with npz.open(f"{ident}.npy", "w", force_zip64=True) as member:
            np.lib.format.write_array(member, np.ascontiguousarray(array).copy(), version=(1, 0),
                                      allow_pickle=False)


def save(obj, path) -> None:
    """Writes `obj` as an archive at `path`: metadata.json, then arrays.npz (itself a stored
    ZIP of NPY members), replacing any previous file atomically."""
    encoded, arrays = metadata_bytes(obj)
    with _replacing(Path(path)) as out, _stored_zip(out) as archive:
        archive.writestr("metadata.json", encoded)
        with archive.open("arrays.npz", "w", force_zip64=True) as payload, _stored_zip(payload) as npz:
            _write_arrays(npz, arrays)


# ---- reading ---------------------------------------------------------------------------------
def _unique_pairs(pairs):
    out = {}
    for key, value in pairs:
        if key in out:
            raise SerializationError(f"Duplicate JSON field {key!r}.")
        out[key] = value
    return out


def _no_constants(value):
    raise SerializationError(f"Nonstandard JSON constant {value!r} is forbidden.")


def _exact_fields(value, expected, what):
    if type(value) is not dict or set(value) != set(expected):
        raise SerializationError(f"Invalid {what} fields; expected {sorted(expected)}.")


def _stored_entries(archive: zipfile.ZipFile, expected: set) -> None:
    infos = archive.infolist()
    names = [info.filename for info in infos]
    if len(names) != len(set(names)) or set(names) != set(expected):
        raise SerializationError("Archive contains duplicate, missing or unexpected entries.")
    for info in infos:
        if info.compress_type != zipfile.ZIP_STORED or info.flag_bits & 1:
            raise SerializationError("Archive entries must be uncompressed and unencrypted.")


def _records(entries, max_array_bytes):
    if type(entries) is not list:
        raise SerializationError("Array records must be a list.")
    out, total = {}, 0
    for index, record in enumerate(entries):
        _exact_fields(record, {"id", "dtype", "shape", "nbytes"}, "array record")
        if record["id"] != f"a{index}":
            raise SerializationError("Array IDs must be unique consecutive identifiers.")
        dtype = _checked_dtype(record["dtype"])
        shape = record["shape"]
        if type(shape) is not list or any(type(n) is not int or not 0 <= n <= np.iinfo(np.intp).max for n in shape):
            raise SerializationError("Array shape must contain nonnegative platform-sized integers.")
        nbytes = math.prod(shape) * dtype.itemsize
        if type(record["nbytes"]) is not int or record["nbytes"] != nbytes or nbytes > np.iinfo(np.intp).max:
            raise SerializationError("Array nbytes does not match its shape and dtype or exceeds the platform limit.")
        total += nbytes
        if max_array_bytes is not None and total > max_array_bytes:
            raise SerializationError("Archive arrays exceed max_array_bytes.")
        out[record["id"]] = (dtype, tuple(shape), nbytes)
    return out


def _read_npy(npz: zipfile.ZipFile, ident: str, record) -> np.ndarray:
    dtype, shape, nbytes = record
    info = npz.getinfo(f"{ident}.npy")
    with npz.open(info) as stream:
        if np.lib.format.read_magic(stream) != (1, 0):
            raise SerializationError("Only NPY version 1.0 is supported by this archive format.")
        got_shape, fortran, got_dtype = np.lib.format.read_array_header_1_0(stream)
        if got_shape != shape or got_dtype != dtype or fortran:
            raise SerializationError(f"NPY header disagrees with metadata for {ident!r}.")
        if info.file_size - stream.tell() != nbytes:
            raise SerializationError(f"Invalid array payload size for {ident!r}.")
        stream.seek(0)
        return np.lib.format.read_array(stream, allow_pickle=False)


def _from_tree(node, npz, records, used, depth=0):
    if depth > _MAX_DEPTH:
        raise SerializationError(f"Archive nesting exceeds {_MAX_DEPTH} levels.")
    if type(node) is not dict or type(node.get("type")) is not str:
        raise SerializationError("Every tree node must have a string type tag.")
    kind = node["type"]
    if kind == "none":
        _exact_fields(node, {"type"}, "none node")
        return None
    if kind in ("bool", "int", "str", "float"):
        _exact_fields(node, {"type", "value"}, "scalar node")
        value = node["value"]
        if type(value) is not {"bool": bool, "int": int, "str": str, "float": str}[kind]:
            raise SerializationError(f"Invalid scalar value for type {kind!r}.")
        if kind == "float":
            converted = float.fromhex(value)
            if converted.hex() != value:
                raise SerializationError("Float values must use canonical hexadecimal strings.")
            return converted
        return value
    if kind in ("list", "tuple", "dict"):
        _exact_fields(node, {"type", "items"}, "container node")
        if type(node["items"]) is not list:
            raise SerializationError("Container items must be a list.")
        if kind == "dict":
            out = {}
            for pair in node["items"]:
                if type(pair) is not list or len(pair) != 2 or type(pair[0]) is not str or pair[0] in out:
                    raise SerializationError("Dictionary entries must have unique string keys.")
                out[pair[0]] = _from_tree(pair[1], npz, records, used, depth + 1)
            return out
        items = [_from_tree(item, npz, records, used, depth + 1) for item in node["items"]]
        return tuple(items) if kind == "tuple" else items
    if kind in ("tensor", "ndarray"):
        _exact_fields(node, {"type", "id", "requires_grad"} if kind == "tensor" else {"type", "id"}, "array node")
        ident = node["id"]
        if type(ident) is not str or ident not in records or ident in used:
            raise SerializationError("Array reference must name a unique existing array ID.")
        used.add(ident)
        array = _read_npy(npz, ident, records[ident])
        if kind == "ndarray":
            return array
        grad = node["requires_grad"]
        if type(grad) is not bool or (grad and records[ident][0].kind != "f"):
            raise SerializationError("Invalid requires_grad flag for serialized Tensor dtype.")
        return torch.from_numpy(np.array(array, copy=True)).requires_grad_(grad)
    raise SerializationError(f"Unknown archive tree node type {kind!r}.")


def load(path, *, max_array_bytes=None):
    """Reads an archive written by `save` or by the reference's `namitorch.serialization.save`."""
    if max_array_bytes is not None and (type(max_array_bytes) is not int or max_array_bytes < 0):
        raise TypeError("max_array_bytes must be a nonnegative Python integer or None.")
    try:
        with zipfile.ZipFile(path, "r") as archive:
            _stored_entries(archive, {"metadata.json", "arrays.npz"})
            if archive.getinfo("metadata.json").file_size > _MAX_METADATA_BYTES:
                raise SerializationError("Archive metadata exceeds the 16 MiB format limit.")
            metadata = json.loads(archive.read("metadata.json"), object_pairs_hook=_unique_pairs,
                                  parse_constant=_no_constants)
            _exact_fields(metadata, {"format_version", "tree", "arrays"}, "metadata")
            if type(metadata["format_version"]) is not int or metadata["format_version"] != FORMAT_VERSION:
                raise SerializationError("Unsupported archive format_version.")
            records = _records(metadata["arrays"], max_array_bytes)
            with archive.open("arrays.npz") as payload, zipfile.ZipFile(payload, "r") as npz:
                _stored_entries(npz, {f"{ident}.npy" for ident in records})
                used: set = set()
                result = _from_tree(metadata["tree"], npz, records, used)
                if used != set(records):
                    raise SerializationError("Archive contains unreferenced arrays.")
                return result
    except SerializationError:
        raise
    except (zipfile.BadZipFile, ValueError, TypeError, KeyError, EOFError, OverflowError, RecursionError) as error:
        raise SerializationError(f"Invalid NamiTorch archive: {error}") from error


# ---- optimizer / scaler checkpoints -----------------------------------------------------------
def pack_optimizer(optimizer):
    """optimizer.state_dict() with the state indices as decimal strings
    (namitorch/training/checkpoint.py:59-64)."""
    if optimizer is None:
        return None
    state = optimizer.state_dict()
    state["state"] = {str(index): values for index, values in state["state"].items()}
    return state


def unpack_optimizer(state):
    """Inverse of pack_optimizer, with the reference's checks (checkpoint.py:67-77)."""
    if not isinstance(state, dict) or not isinstance(state.get("state"), dict):
        raise SerializationError("Invalid checkpoint optimizer state.")
    restored = dict(state)
    values = {}
    for key, value in state["state"].items():
        if type(key) is not str or not key.isascii() or not key.isdecimal() or str(int(key)) != key:
            raise SerializationError("Optimizer state indices must be canonical nonnegative integer strings.")
        values[int(key)] = value
    restored["state"] = values
    return restored


def _counter(value, name):
    if isinstance(value, bool) or not isinstance(value, Integral) or value < 0:
        raise ValueError(f"{name} must be a nonnegative integer.")
    return int(value)


def reference_optimizer_type(optimizer) -> str | None:
    """The reference's class path for this optimizer's kind ("namitorch.optim.adam.AdamW"),
    which the reference's load_checkpoint compares with its own optimizer."""
    if optimizer is None:
        return None
    return f"namitorch.optim.adam.{'AdamW' if getattr(optimizer, '_decoupled_weight_decay', False) else 'Adam'}"


def save_checkpoint(path, optimizer=None, scaler=None, *, model_state=None, parameter_names=None,
                    scheduler_state=None, rng=None, step=0, epoch=0, config=None, cumulative_tokens=0) -> None:
    """Writes a checkpoint with the reference's fields (checkpoint.py:80-110).

    `model_state` is the model's state dict (name -> tensor); `parameter_names` lists, per
    parameter group, the model names of the group's parameters (the reference checks them
    against its model when it loads). The optimizer is stored as the reference's AdamW /
    Adam (`optimizer_type`), whose state_dict format this package keeps. `rng` is stored as
    given (the reference restores it only with restore_rng=True)."""
    if scaler is not None and not hasattr(scaler, "state_dict"):
        raise TypeError("scaler must be a GradScaler or None.")
    checkpoint = {
        "checkpoint_version": CHECKPOINT_VERSION,
        "model": {} if model_state is None else dict(model_state),
        "optimizer": pack_optimizer(optimizer),
        "optimizer_type": reference_optimizer_type(optimizer),
        "optimizer_parameter_names": parameter_names,
        "scheduler": scheduler_state,
        "rng": rng,
        "step": _counter(step, "step"),
        "epoch": _counter(epoch, "epoch"),
        "config": config,
        "cumulative_tokens": _counter(cumulative_tokens, "cumulative_tokens"),
    }
    if scaler is not None:
        checkpoint["scaler"] = scaler.state_dict()
    save(checkpoint, path)


def load_checkpoint(path, optimizer=None, scaler=None, *, parameter_names=None, max_array_bytes=None) -> dict:
    """Reads a checkpoint written by the reference's save_checkpoint or by save_checkpoint
    above, restores `optimizer` and `scaler` from it, and returns the remaining fields
    (step, epoch, cumulative_tokens, config, model state, scheduler state, rng)."""
    checkpoint = load(path, max_array_bytes=max_array_bytes)
    if type(checkpoint) is not dict or set(checkpoint) not in (_CHECKPOINT_KEYS, _CHECKPOINT_KEYS | {"scaler"}):
        raise SerializationError("Invalid checkpoint fields.")
    if type(checkpoint["checkpoint_version"]) is not int or checkpoint["checkpoint_version"] != CHECKPOINT_VERSION:
        raise SerializationError("Unsupported checkpoint_version.")
    info = {name: _counter(checkpoint[name], name) for name in ("step", "epoch", "cumulative_tokens")}
    info.update(config=checkpoint["config"], model=checkpoint["model"], scheduler=checkpoint["scheduler"],
                rng=checkpoint["rng"])
    if optimizer is not None:
        if checkpoint["optimizer_type"] != reference_optimizer_type(optimizer):
            raise ValueError("Checkpoint optimizer type does not match the supplied optimizer.")
        if parameter_names is not None and checkpoint["optimizer_parameter_names"] != parameter_names:
            raise ValueError("Checkpoint optimizer parameter names or group order do not match the model.")
        optimizer.load_state_dict(unpack_optimizer(checkpoint["optimizer"]))
    if scaler is not None:
        if "scaler" not in checkpoint:
            raise SerializationError("Checkpoint has no GradScaler state.")
        scaler.load_state_dict(checkpoint["scaler"])
    return info


__all__ = ["FORMAT_VERSION", "SerializationError", "save", "load", "metadata_bytes", "pack_optimizer",
           "unpack_optimizer", "save_checkpoint", "load_checkpoint", "reference_optimizer_type"]
