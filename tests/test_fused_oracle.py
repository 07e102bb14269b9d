"""The fused-activation oracle against outputs of the reference's own CPU path and autograd
(tests/golden/make_fused_golden.py): bit for bit, except gelu(tanh), where the reference
cubes with a power (one rounding) and the kernels multiply (two): within 4 float32 ulps."""
import numpy as np
import pytest

from conftest import REPO
from oracle import activations as A

G = np.load(REPO / "tests" / "golden" / "fused.npz")


def same(got, want, ulps=0):
    got, want = np.asarray(got, np.float32), np.asarray(want, np.float32)
    assert got.shape == want.shape
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    if ulps == 0:
        assert np.array_equal(got[~nan], want[~nan])
        assert np.array_equal(np.signbit(got[~nan]), np.signbit(want[~nan]))
    else:
        fin = ~nan & np.isfinite(want)
        assert np.array_equal(got[~nan & ~fin], want[~nan & ~fin])
        tol = ulps * np.spacing(np.abs(want[fin]).astype(np.float32))
        assert np.all(np.abs(got[fin] - want[fin]) <= tol)


@pytest.mark.parametrize("name", ["sigmoid", "silu", "gelu_tanh"])
def test_unary_forward_and_gradient(name):
    x, g = G["x"], G["g"]
    ulps = 4 if name == "gelu_tanh" else 0
    y = A.apply(name, (x,))
    same(y, G[f"{name}_y"], ulps)
    saved = y if name == "sigmoid" else x
    same(A.apply(f"{name}_backward", (saved, g)), G[f"{name}_dx"], ulps)


def test_swiglu():
    x, up, g = G["x"], G["up"], G["g"]
    same(A.apply("swiglu", (x, up)), G["swiglu_y"])
    dgate, dup = A.apply("swiglu_backward", (x, up, g))
    same(dgate, G["swiglu_dgate"])
    same(dup, G["swiglu_dup"])


@pytest.mark.parametrize("name", ["relu", "sigmoid", "silu", "gelu_tanh"])
def test_bias_activation(name):
    x, bias, g = G["x"].reshape(4, 16), G["bias"], G["g"].reshape(4, 16)
    ulps = 4 if name == "gelu_tanh" else 0
    same(A.apply(f"bias_{name}", (x, bias)), G[f"bias_{name}_y"], ulps)
    same(A.apply(f"bias_{name}_backward", (x, bias, g)), G[f"bias_{name}_dx"], ulps)


@pytest.mark.parametrize("tag,lo,hi", [("min", -0.5, None), ("max", None, 0.75), ("both", -0.5, 0.75)])
def test_clamp(tag, lo, hi):
    x, g = G["x"], G["g"]
    same(A.apply("clamp", (x, lo, hi)), G[f"clamp_{tag}_y"])
    same(A.apply("clamp_backward", (x, lo, hi, g)), G[f"clamp_{tag}_dx"])


def test_nan_bound_poisons_clamp():
    x = np.array([1.0, -2.0], np.float32)
    assert np.isnan(A.apply("clamp", (x, np.float32(np.nan), None))).all()
    assert np.isnan(A.apply("clamp_backward", (x, None, np.float32(np.nan), x))).all()
