"""Generates ``norm.npz`` by running the reference's CPU layer_norm / rms_norm and autograd.

Cases (float32): layer_norm of [6, 10, 48] with weight and bias, rms_norm of [5, 7, 33]
with weight; for each, the output, an upstream gradient and the gradients the reference's
autograd returns for the input, weight and bias.

Usage (needs the reference checkout; not run by the tests):
    python tests/golden/make_norm_golden.py /path/to/reference
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    import namitorch as nt
    from namitorch.nn import functional as F

    rng = np.random.default_rng(5)
    out = {}
    x = (rng.normal(0, 2, (6, 10, 48)) + 3).astype(np.float32)
    w = rng.normal(1, 0.2, 48).astype(np.float32)
    b = rng.normal(0, 0.2, 48).astype(np.float32)
    g = rng.normal(0, 1, x.shape).astype(np.float32)
    xt, wt, bt = (nt.tensor(a, requires_grad=True) for a in (x, w, b))
    y = F.layer_norm(xt, 48, wt, bt, eps=1e-5)
    y.backward(nt.tensor(g))
    out.update(layer_x=x, layer_w=w, layer_b=b, layer_g=g, layer_y=np.asarray(y._data),
               layer_dx=np.asarray(xt.grad._data), layer_dw=np.asarray(wt.grad._data),
               layer_db=np.asarray(bt.grad._data))
    x = rng.normal(0, 1.5, (5, 7, 33)).astype(np.float32)
    w = rng.normal(1, 0.2, 33).astype(np.float32)
    g = rng.normal(0, 1, x.shape).astype(np.float32)
    xt, wt = nt.tensor(x, requires_grad=True), nt.tensor(w, requires_grad=True)
    y = F.rms_norm(xt, 33, wt, eps=1e-6)
    y.backward(nt.tensor(g))
    out.update(rms_x=x, rms_w=w, rms_g=g, rms_y=np.asarray(y._data), rms_dx=np.asarray(xt.grad._data),
               rms_dw=np.asarray(wt.grad._data))
    np.savez(HERE / "norm.npz", **out)
    print("wrote norm.npz", sorted(out))


if __name__ == "__main__":
    main(sys.argv[1])
