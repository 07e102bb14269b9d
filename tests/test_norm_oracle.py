"""The normalization oracle against the reference's CPU layer_norm / rms_norm and autograd.

The oracle follows the reference's fused kernels (anchored two-moment statistics); the
reference's CPU path computes the same quantities with other float32 sums, so the two agree
to float32 rounding: within 4e-7 of each array's largest magnitude per summed row element.
"""
import numpy as np
import pytest

from conftest import REPO
from oracle import normalization as O

GOLDEN = np.load(REPO / "tests" / "golden" / "norm.npz")


def _close(a, b, rows=1):
    scale = float(np.max(np.abs(b)))
    assert float(np.max(np.abs(a - b))) <= 4e-7 * scale * max(1, rows)


def test_layer_norm_matches_reference():
    d = GOLDEN
    y, st = O.forward(d["layer_x"], d["layer_w"], d["layer_b"], 1e-5, True)
    dx, dw, db = O.backward(d["layer_x"], d["layer_w"], d["layer_g"], st, True)
    _close(y, d["layer_y"])
    _close(dx, d["layer_dx"])
    _close(dw, d["layer_dw"], rows=60)
    _close(db, d["layer_db"], rows=60)


def test_rms_norm_matches_reference():
    d = GOLDEN
    y, st = O.forward(d["rms_x"], d["rms_w"], None, 1e-6, False)
    dx, dw, _ = O.backward(d["rms_x"], d["rms_w"], d["rms_g"], st, False)
    assert np.all(st[:, 0] == 0)
    _close(y, d["rms_y"])
    _close(dx, d["rms_dx"])
    _close(dw, d["rms_dw"], rows=35)
