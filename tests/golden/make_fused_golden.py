"""Generates ``fused.npz`` by running the reference's CPU activations and their autograd.

Inputs (float32): one vector of 64 values holding ±0, ±inf, NaN, values beyond |x| = 20 and a
seeded normal spread, and an upstream gradient. For each of sigmoid, silu and gelu(tanh):
the forward and the input gradient. swiglu: the output and both operand gradients. The bias
activations (relu, sigmoid, silu, gelu tanh) on [4, 16] with a [16] bias: the output and the
input gradient (the elementwise local gradient). clamp with a minimum, a maximum and both:
the output and the input gradient.

Usage (needs the reference checkout; not run by the tests):
    python tests/golden/make_fused_golden.py /path/to/reference
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    import namitorch as nt
    import namitorch.nn.functional as F

    rng = np.random.default_rng(5)
    x = rng.normal(0, 3, 64).astype(np.float32)
    x[:12] = [0.0, -0.0, np.inf, -np.inf, np.nan, 25.0, -25.0, 20.0, -20.0, 19.5, -19.5, 1e-30]
    g = rng.normal(0, 1, 64).astype(np.float32)
    out = {"x": x, "g": g}

    def grad_of(fn, *arrays):
        ts = [nt.tensor(a, requires_grad=True) for a in arrays]
        y = fn(*ts)
        y.backward(nt.tensor(g.reshape(y.shape)))
        return np.asarray(y._data), [np.asarray(t.grad._data) for t in ts]

    for name, fn in (("sigmoid", lambda t: t.sigmoid()), ("silu", lambda t: t.silu()),
                     ("gelu_tanh", lambda t: t.gelu("tanh"))):
        y, (dx,) = grad_of(fn, x)
        out[f"{name}_y"], out[f"{name}_dx"] = y, dx

    up = rng.normal(0, 1, 64).astype(np.float32)
    out["up"] = up
    y, (dgate, dup) = grad_of(F.swiglu, x, up)
    out["swiglu_y"], out["swiglu_dgate"], out["swiglu_dup"] = y, dgate, dup

    xb = x.reshape(4, 16)
    bias = rng.normal(0, 1, 16).astype(np.float32)
    out["bias"] = bias
    for act in ("relu", "sigmoid", "silu", "gelu"):
        name = "gelu_tanh" if act == "gelu" else act
        y, (dx, _) = grad_of(lambda t, b, a=act: F.bias_activation(t, b, a, approximation="tanh"), xb, bias)
        out[f"bias_{name}_y"], out[f"bias_{name}_dx"] = y, dx

    for tag, lo, hi in (("min", -0.5, None), ("max", None, 0.75), ("both", -0.5, 0.75)):
        y, (dx,) = grad_of(lambda t, lo=lo, hi=hi: t.clamp(None if lo is None else np.float32(lo),
                                                               None if hi is None else np.float32(hi)), x)
        out[f"clamp_{tag}_y"], out[f"clamp_{tag}_dx"] = y, dx

    np.savez(HERE / "fused.npz", **out)
    print("wrote fused.npz", sorted(out))


if __name__ == "__main__":
    main(sys.argv[1])
