"""Checkpoint archives against the reference's own files (CPU).

``tests/golden/archive_ref.zip`` and ``checkpoint_ref.zip`` were written by the reference's
``namitorch.serialization.save`` / ``namitorch.training.checkpoint.save_checkpoint``
(``tests/golden/make_checkpoint_golden.py``). The reader must return every value, and the
writer must reproduce the reference's ``metadata.json`` byte for byte from the loaded tree.
"""
import hashlib
import json
import zipfile

import numpy as np
import pytest
import torch

from conftest import REPO
from namitorch_b200 import checkpoint as C

GOLDEN = REPO / "tests" / "golden"
EXPECT = json.loads((GOLDEN / "checkpoint_expect.json").read_text())


def sha(a) -> str:
    a = a.detach().numpy() if isinstance(a, torch.Tensor) else a
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _metadata(path) -> bytes:
    with zipfile.ZipFile(path) as z:
        return z.read("metadata.json")


def test_reads_every_node_kind_of_a_reference_archive():
    obj = C.load(GOLDEN / "archive_ref.zip")
    assert obj["none"] is None and obj["flag"] is True and obj["count"] == -7 and obj["ratio"] == 0.1
    assert obj["text"] == "zéro" and obj["items"] == [1, 2.5, "x"] and obj["pair"] == (3, (4.0, None))
    assert obj["nested"] == {"k": [{"deep": False}]}
    np.testing.assert_array_equal(obj["f32"], np.arange(6, dtype=np.float32).reshape(2, 3) / 7)
    assert obj["f16"].dtype == np.float16 and obj["i64"].tolist() == [-1, 2 ** 40] and obj["u8"].tolist() == [0, 255]
    assert obj["b"].dtype == np.bool_ and obj["empty"].shape == (0, 3) and obj["f64"][0] == np.pi
    t = obj["tensor"]
    assert isinstance(t, torch.Tensor) and t.dtype == torch.float32 and not t.requires_grad
    assert t.tolist() == [[1.0, -1.0]]


@pytest.mark.parametrize("name", ["archive_ref.zip", "checkpoint_ref.zip"])
def test_writer_reproduces_reference_metadata_bytes(name, tmp_path):
    obj = C.load(GOLDEN / name)
    encoded, arrays = C.metadata_bytes(obj)
    assert encoded == _metadata(GOLDEN / name)
    out = tmp_path / name
    C.save(obj, out)
    assert _metadata(out) == _metadata(GOLDEN / name)
    again = C.load(out)
    _, arrays2 = C.metadata_bytes(again)
    for (i1, a1), (i2, a2) in zip(arrays, arrays2):
        assert i1 == i2 and a1.dtype == a2.dtype and np.array_equal(a1, a2)


def test_reference_checkpoint_fields_and_optimizer_state():
    ck = C.load(GOLDEN / "checkpoint_ref.zip")
    assert ck["checkpoint_version"] == 1 and ck["step"] == 3 and ck["epoch"] == 1
    assert ck["cumulative_tokens"] == 12345 and ck["config"] == {"lr": 1e-2, "note": "tiny"}
    assert ck["optimizer_type"] == "namitorch.optim.adam.AdamW"
    assert ck["optimizer_parameter_names"] == [["a.weight", "b.weight"], ["a.bias", "b.bias"]]
    for name in EXPECT["names"]:
        assert sha(ck["model"][name]) == EXPECT["model_sha"][name]
    opt = C.unpack_optimizer(ck["optimizer"])
    assert set(opt["state"]) == {0, 1, 2, 3}
    for k, values in opt["state"].items():
        want = EXPECT["state"][str(k)]
        assert values["step"] == want["step"]
        assert sha(values["exp_avg"]) == want["exp_avg_sha"] and sha(values["exp_avg_sq"]) == want["exp_avg_sq_sha"]
    scaler = ck["scaler"]
    assert scaler["scale"] == float.fromhex(EXPECT["scaler"]["scale"]) and scaler["growth_tracker"] == 0


def test_round_trip_of_torch_and_numpy_values(tmp_path):
    obj = {"w": torch.arange(12, dtype=torch.float32).reshape(3, 4).requires_grad_(True),
           "i": torch.tensor([1, 2], dtype=torch.int64), "h": torch.tensor([0.5], dtype=torch.float16),
           "n": np.ones((2, 2), np.float64), "t": (1, "a", None, [0.25])}
    C.save(obj, tmp_path / "x.zip")
    back = C.load(tmp_path / "x.zip")
    assert back["w"].requires_grad and torch.equal(back["w"].detach(), obj["w"].detach())
    assert back["i"].dtype == torch.int64 and back["h"].dtype == torch.float16
    assert np.array_equal(back["n"], obj["n"]) and back["t"] == (1, "a", None, [0.25])


def test_format_rules_are_enforced(tmp_path):
    with pytest.raises(C.SerializationError, match="bfloat16"):
        C.save({"x": torch.zeros(2, dtype=torch.bfloat16)}, tmp_path / "a.zip")
    cyclic = []
    cyclic.append(cyclic)
    with pytest.raises(C.SerializationError, match="cyclic"):
        C.save(cyclic, tmp_path / "b.zip")
    with pytest.raises(TypeError, match="string keys"):
        C.save({1: 2}, tmp_path / "c.zip")
    with pytest.raises(TypeError, match="Cannot serialize set"):
        C.save({"s": {1}}, tmp_path / "d.zip")
    with pytest.raises(C.SerializationError, match="complex"):
        C.save({"z": np.zeros(2, np.complex64)}, tmp_path / "e.zip")
    # A compressed entry and an unexpected entry are rejected on load.
    bad = tmp_path / "f.zip"
    with zipfile.ZipFile(bad, "w", compression=zipfile.ZIP_DEFLATED) as z:
        z.writestr("metadata.json", _metadata(GOLDEN / "archive_ref.zip"))
        z.writestr("arrays.npz", b"")
    with pytest.raises(C.SerializationError, match="uncompressed"):
        C.load(bad)
    with pytest.raises(C.SerializationError, match="max_array_bytes"):
        C.load(GOLDEN / "checkpoint_ref.zip", max_array_bytes=16)
    with pytest.raises(C.SerializationError, match="canonical"):
        C.unpack_optimizer({"state": {"01": {}}})
