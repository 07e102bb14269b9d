"""Generates the checkpoint fixtures in this directory by running the reference itself.

``namitorch.training.checkpoint.save_checkpoint`` of the reference writes
``checkpoint_ref.zip``: a two-linear-layer model, an AdamW (two parameter groups) after
three NumPy steps with seeded gradients, and a GradScaler after an overflow step. The
reference's ``namitorch.serialization.save`` also writes ``archive_ref.zip`` from a small
object of every node kind the format has (None, bool, int, float, str, list, tuple, dict,
ndarray of several dtypes, Tensor). ``checkpoint_expect.json`` records what the tests need
to check a reader against: the step counts, hex floats of sampled state values and SHA-256
checksums of every saved array, and the fourth step's inputs (gradients seed) so that a GPU
test can continue the run from the checkpoint.

Usage (needs the reference checkout; not run by the tests):
    python tests/golden/make_checkpoint_golden.py /path/to/reference
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

SHAPES = [(16, 8), (16,), (4, 16), (4,)]
NAMES = ["a.weight", "a.bias", "b.weight", "b.bias"]
LR, BETAS, EPS, WD = 1e-2, (0.9, 0.999), 1e-8, 0.1


def grads_for(step: int) -> list[np.ndarray]:
    rng = np.random.default_rng(1000 + step)
    return [rng.normal(0.0, 0.05, s).astype(np.float32) for s in SHAPES]


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    import namitorch as nt
    from namitorch import nn
    from namitorch.amp import GradScaler
    from namitorch.optim import AdamW
    from namitorch.serialization import save
    from namitorch.training.checkpoint import save_checkpoint

    class Tiny(nn.Module):
        def __init__(self):
            super().__init__()
            self.a = nn.Linear(8, 16)
            self.b = nn.Linear(16, 4)

    rng = np.random.default_rng(7)
    model = Tiny()
    params = dict(model.named_parameters())
    assert list(params) == NAMES, list(params)
    for name, shape in zip(NAMES, SHAPES):
        params[name]._data[...] = rng.normal(0.0, 0.1, shape).astype(np.float32)
    initial = {name: np.asarray(params[name]._data).copy() for name in NAMES}
    weights = [params["a.weight"], params["b.weight"]]
    biases = [params["a.bias"], params["b.bias"]]
    opt = AdamW([{"params": weights, "weight_decay": WD}, {"params": biases, "weight_decay": 0.0}],
                lr=LR, betas=BETAS, eps=EPS, fused=False)
    order = ["a.weight", "b.weight", "a.bias", "b.bias"]   # registration order: group by group
    for step in range(3):
        for name, g in zip(NAMES, grads_for(step)):
            params[name]._grad = nt.tensor(g)
        opt.step()
    # One AMP round whose gradients overflow: unscale_, a skipped step, update -> scale 512.
    scaler = GradScaler(init_scale=1024.0, growth_interval=3)
    for name, g in zip(NAMES, grads_for(99)):
        g = g.copy()
        if name == "b.bias":
            g[1] = np.inf
        params[name]._grad = nt.tensor(g)
    scaler.scale(nt.tensor(np.float32(1.0)))
    scaler.unscale_(opt)
    assert not scaler.step(opt)
    scaler.update()
    assert scaler.get_scale() == 512.0
    save_checkpoint(HERE / "checkpoint_ref.zip", model, opt, step=3, epoch=1, config={"lr": LR, "note": "tiny"},
                    cumulative_tokens=12345, scaler=scaler)

    sample = {
        "none": None, "flag": True, "count": -7, "ratio": 0.1, "text": "zéro", "items": [1, 2.5, "x"],
        "pair": (3, (4.0, None)), "nested": {"k": [{"deep": False}]},
        "f32": np.arange(6, dtype=np.float32).reshape(2, 3) / 7,
        "f16": np.array([1.5, -2.0, 65504.0], dtype=np.float16),
        "f64": np.array([np.pi], dtype=np.float64), "i64": np.array([-1, 2**40], dtype=np.int64),
        "u8": np.array([0, 255], dtype=np.uint8), "b": np.array([True, False]),
        "empty": np.zeros((0, 3), dtype=np.float32), "tensor": nt.tensor(np.array([[1.0, -1.0]], dtype=np.float32)),
    }
    save(sample, HERE / "archive_ref.zip")

    sd = opt.state_dict()
    expect = {
        "names": NAMES, "shapes": [list(s) for s in SHAPES], "registration_order": order,
        "options": {"lr": LR, "betas": list(BETAS), "eps": EPS, "weight_decay": WD},
        "initial_sha": {n: sha(initial[n]) for n in NAMES},
        "model_sha": {n: sha(np.asarray(params[n]._data)) for n in NAMES},
        "state": {str(k): {"step": v["step"], "exp_avg_sha": sha(np.asarray(v["exp_avg"]._data)),
                           "exp_avg_sq_sha": sha(np.asarray(v["exp_avg_sq"]._data)),
                           "exp_avg_first": float(np.asarray(v["exp_avg"]._data).reshape(-1)[0]).hex()}
                  for k, v in sd["state"].items()},
        "scaler": {k: (float(v).hex() if isinstance(v, float) else v) for k, v in scaler.state_dict().items()},
        "grad_seed_base": 1000, "next_step": 3,
    }
    # The fourth step, run by the reference from the same state, for the resume test.
    for name, g in zip(NAMES, grads_for(3)):
        params[name]._grad = nt.tensor(g)
    opt.step()
    expect["after_step4_sha"] = {n: sha(np.asarray(params[n]._data)) for n in NAMES}
    (HERE / "checkpoint_expect.json").write_text(json.dumps(expect, indent=1) + "\n")
    print("wrote checkpoint_ref.zip, archive_ref.zip, checkpoint_expect.json")


if __name__ == "__main__":
    main(sys.argv[1])
