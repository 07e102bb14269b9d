"""Generates ``softmax.npz`` by running the reference's CPU softmax and its autograd.

Cases (float32): plain softmax over the last dimension of [4, 7, 33] with some -inf scores;
masked softmax of [2, 3, 5, 40] scores with a [5, 40] boolean mask broadcast over batch and
heads (the reference's attention path: masked_fill(-inf) then softmax); causal softmax of
[2, 5, 9] scores with query_position_offset 2, and causal softmax of [2, 6, 40] scores whose
blocked positions hold NaN and +inf. For each, the upstream gradient and the
gradient the reference's autograd returns for the scores.

Usage (needs the reference checkout; not run by the tests):
    python tests/golden/make_softmax_golden.py /path/to/reference
"""
from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    import namitorch as nt

    rng = np.random.default_rng(11)
    out = {}

    def run(name, x, blocked):
        t = nt.tensor(x, requires_grad=True)
        scores = t.masked_fill(nt.tensor(blocked), -float("inf")) if blocked is not None else t
        y = scores.softmax(-1)
        g = rng.normal(0, 1, x.shape).astype(np.float32)
        y.backward(nt.tensor(g))
        out[f"{name}_x"] = x
        out[f"{name}_y"] = np.asarray(y._data)
        out[f"{name}_g"] = g
        out[f"{name}_dx"] = np.asarray(t.grad._data)

    x = rng.normal(0, 3, (4, 7, 33)).astype(np.float32)
    x[0, 1, 5] = -np.inf
    x[2, 3, :10] = -np.inf
    run("plain", x, None)

    x = rng.normal(0, 2, (2, 3, 5, 40)).astype(np.float32)
    mask = rng.random((5, 40)) < 0.7
    mask[:, 0] = True
    out["masked_mask"] = mask
    run("masked", x, np.broadcast_to(~mask, x.shape).copy())

    x = rng.normal(0, 2, (2, 5, 9)).astype(np.float32)
    offset = 2
    allowed = np.arange(9)[None, :] - min(offset, 9) <= np.arange(5)[:, None]
    out["causal_offset"] = np.array(offset)
    run("causal", x, np.broadcast_to(~allowed, x.shape).copy())

    # The same causal rule with NaN and +inf planted in the blocked (future) positions: the
    # reference fills them with -inf before the softmax, so they change nothing.
    x = rng.normal(0, 2, (2, 6, 40)).astype(np.float32)
    allowed = np.arange(40)[None, :] - min(offset, 40) <= np.arange(6)[:, None]
    blocked = np.broadcast_to(~allowed, x.shape)
    poison = np.where(rng.random(x.shape) < 0.5, np.float32(np.nan), np.float32(np.inf))
    x = np.where(blocked, poison, x).astype(np.float32)
    run("causal_poisoned", x, blocked.copy())

    np.savez(HERE / "softmax.npz", **out)
    print("wrote softmax.npz", sorted(out))


if __name__ == "__main__":
    main(sys.argv[1])
