"""GPU parity of the fused elementwise activations (nt_fused_elementwise) through the seam.

float32 results within 4e-6 relative plus 2e-6 of the array's largest magnitude of the
oracle (the device's expf / tanhf against NumPy's, a few float32 ulps, and the derivative
sums that cancel near zero); float16 / bfloat16 outputs within one unit of the stored type.
"""
import zlib

import numpy as np
import pytest
import torch

from conftest import REPO
from namitorch_b200.backends import enable_fused_kernels, get_backend, try_fused
from namitorch_b200.backends.fused import OPERATIONS
from oracle import activations as A
from oracle.casts import round_to_bf16

pytestmark = pytest.mark.gpu
G = np.load(REPO / "tests" / "golden" / "fused.npz")
TORCH = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _store(x, dt):
    x = np.asarray(x, np.float32)
    if dt == "bf16":
        return round_to_bf16(x)
    if dt == "f16":
        return x.astype(np.float16).astype(np.float32)
    return x


def _close(got, want, dt="f32"):
    got = got.float().cpu().numpy() if isinstance(got, torch.Tensor) else np.asarray(got)
    want = np.asarray(want, np.float32)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan)
    inf = np.isinf(want)
    assert np.array_equal(got[inf], want[inf])
    fin = ~nan & ~inf
    if not fin.any():
        return
    scale = float(np.max(np.abs(want[fin])))
    if dt == "f32":
        err = np.abs(got[fin] - want[fin])
        assert np.all(err <= 4e-6 * np.abs(want[fin]) + 2e-6 * scale), f"max error {float(np.max(err))} at scale {scale}"
    else:
        unit = 2.0 ** (-7 if dt == "bf16" else -10)
        np.testing.assert_allclose(got[fin], want[fin], rtol=unit, atol=unit * 1e-2 * scale + 1e-6)


def _k():
    return get_backend(torch.zeros(1, device="cuda")).fused


def _t(a, dt="f32"):
    return None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda().to(TORCH[dt])


@pytest.mark.parametrize("name", ["sigmoid", "silu", "gelu_tanh"])
def test_reference_golden_unary(cuda_device, name):
    x, g = G["x"], G["g"]
    y = _k().run(name, (_t(x),))
    _close(y, G[f"{name}_y"])
    saved = G[f"{name}_y"] if name == "sigmoid" else x
    _close(_k().run(f"{name}_backward", (_t(saved), _t(g))), G[f"{name}_dx"])


def test_reference_golden_swiglu_bias_clamp(cuda_device):
    x, g, up, bias = G["x"], G["g"], G["up"], G["bias"]
    _close(_k().run("swiglu", (_t(x), _t(up))), G["swiglu_y"])
    dgate, dup = _k().run("swiglu_backward", (_t(x), _t(up), _t(g)))
    _close(dgate, G["swiglu_dgate"])
    _close(dup, G["swiglu_dup"])
    xb, gb = x.reshape(4, 16), g.reshape(4, 16)
    for name in ("relu", "sigmoid", "silu", "gelu_tanh"):
        _close(_k().run(f"bias_{name}", (_t(xb), _t(bias))), G[f"bias_{name}_y"])
        _close(_k().run(f"bias_{name}_backward", (_t(xb), _t(bias), _t(gb))), G[f"bias_{name}_dx"])
    for tag, lo, hi in (("min", -0.5, None), ("max", None, 0.75), ("both", -0.5, 0.75)):
        tlo = None if lo is None else torch.tensor(lo, dtype=torch.float32, device="cuda")
        thi = None if hi is None else torch.tensor(hi, dtype=torch.float32, device="cuda")
        _close(_k().run("clamp", (_t(x), tlo, thi)), G[f"clamp_{tag}_y"])
        _close(_k().run("clamp_backward", (_t(x), tlo, thi, _t(g))), G[f"clamp_{tag}_dx"])


def _operands(name, shape, dt, rng):
    """Stored (rounded) float32 operands of `name` and their tensors."""
    x = _store(rng.normal(0, 3, shape), dt)
    if name.startswith("bias_"):
        b = _store(rng.normal(0, 1, shape[-1]), dt)
        ops = [x, b] + ([_store(rng.normal(0, 1, shape), dt)] if name.endswith("_backward") else [])
    elif name.startswith("clamp"):
        bounds = [np.float32(_store([-0.7], dt)[0]), np.float32(_store([1.3], dt)[0])]
        ops = [x] + bounds + ([_store(rng.normal(0, 1, shape), dt)] if name.endswith("_backward") else [])
    elif name == "sigmoid_backward":
        ops = [_store(A.sigmoid(x), dt), _store(rng.normal(0, 1, shape), dt)]
    else:
        arity = {"swiglu": 2, "swiglu_backward": 3}.get(name, 2 if name.endswith("_backward") else 1)
        ops = [x] + [_store(rng.normal(0, 1, shape), dt) for _ in range(arity - 1)]
    tensors = []
    for k, a in enumerate(ops):
        if name.startswith("clamp") and k in (1, 2):
            tensors.append(torch.tensor(float(a), dtype=TORCH[dt], device="cuda"))
        else:
            tensors.append(_t(a, dt))
    return ops, tensors


SHAPES = [(7,), (8, 64), (3, 1000), (5, 333), (2, 4096)]


@pytest.mark.parametrize("dt", list(TORCH))
@pytest.mark.parametrize("name", sorted(OPERATIONS))
def test_every_operation_shape_and_dtype_matches_oracle(cuda_device, name, dt):
    rng = np.random.default_rng(zlib.crc32(f"{name}/{dt}".encode()))
    for shape in SHAPES:
        ops, tensors = _operands(name, shape, dt, rng)
        got = _k().run(name, tuple(tensors))
        assert got is not None, (name, shape)
        want = A.apply(name, tuple(ops))
        if name == "swiglu_backward":
            for g_, w_ in zip(got, want):
                _close(g_, _store(w_, dt), dt)
        else:
            assert got.dtype == TORCH[dt] and got.shape == tensors[0].shape
            _close(got, _store(want, dt), dt)


def test_unaligned_operands_take_the_element_path(cuda_device):
    rng = np.random.default_rng(3)
    x = rng.normal(0, 3, 1001).astype(np.float32)
    g = rng.normal(0, 1, 1001).astype(np.float32)
    flat = torch.empty(1002, device="cuda")
    tx = flat[1:]
    tx.copy_(torch.from_numpy(x))
    assert tx.data_ptr() % 16 != 0
    _close(_k().run("gelu_tanh_backward", (tx, _t(g))), A.apply("gelu_tanh_backward", (x, g)))
    xb = x[:1000].reshape(10, 100)
    base = torch.empty(1001, device="cuda")
    txb = base[1:].view(10, 100)
    txb.copy_(torch.from_numpy(xb))
    b = rng.normal(0, 1, 100).astype(np.float32)
    _close(_k().run("bias_silu", (txb, _t(b))), A.apply("bias_silu", (xb, b)))


def test_special_values(cuda_device):
    x = np.array([np.nan, np.inf, -np.inf, 0.0, -0.0, 25.0, -25.0, 88.0, -88.0, -104.0], np.float32)
    tx = _t(x)
    y = _k().run("silu", (tx,)).cpu().numpy()
    assert np.isnan(y[0]) and y[1] == np.inf and y[2] == 0.0
    y = _k().run("gelu_tanh", (tx,)).cpu().numpy()
    assert y[5] == 25.0 and y[6] == 0.0 and np.signbit(y[6])
    r = _k().run("bias_relu_backward", (tx, torch.zeros(10, device="cuda"), torch.ones(10, device="cuda")))
    r = r.cpu().numpy()
    assert np.isnan(r[0]) and r[1] == 1.0 and r[2] == 0.0 and r[3] == 0.0
    s = _k().run("sigmoid", (tx,)).cpu().numpy()
    assert s[1] == 1.0 and s[2] == 0.0 and 0.0 <= s[9] < 1e-44
    c = _k().run("clamp", (tx, torch.tensor(-1.0, device="cuda"), None)).cpu().numpy()
    assert np.isnan(c[0]) and c[1] == np.inf and c[2] == -1.0
    c = _k().run("clamp", (tx, torch.tensor(float("nan"), device="cuda"), None)).cpu().numpy()
    assert np.isnan(c).all()


def test_large_tensor_grid_stride(cuda_device):
    rows, width = 4096, 3072
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1)
    x = torch.randn(rows, width, device="cuda", generator=gen) * 3
    b = torch.randn(width, device="cuda", generator=gen)
    g = torch.randn(rows, width, device="cuda", generator=gen)
    y = _k().run("bias_gelu_tanh", (x, b))
    d = _k().run("bias_gelu_tanh_backward", (x, b, g))
    sel = torch.arange(0, rows, 97, device="cuda")
    xs, gs = x[sel].cpu().numpy(), g[sel].cpu().numpy()
    _close(y[sel], A.apply("bias_gelu_tanh", (xs, b.cpu().numpy())))
    _close(d[sel], A.apply("bias_gelu_tanh_backward", (xs, b.cpu().numpy(), gs)))


def test_declines_empty_and_switch(cuda_device):
    x = torch.randn(4, 8, device="cuda")
    k = _k()
    assert k.run("tanh", (x,)) is None                                   # not a fused operation
    assert k.run("silu", (x.double(),)) is None                          # dtype
    assert k.run("silu", (x.t(),)) is None                               # not contiguous
    assert k.run("silu", (x, x)) is None                                 # arity
    assert k.run("swiglu", (x, x.half())) is None                        # mixed dtypes
    assert k.run("swiglu", (x, x[:2])) is None                           # shapes
    assert k.run("bias_silu", (x, torch.zeros(4, device="cuda"))) is None
    assert k.run("clamp", (x, None, None)) is None                       # no bound
    assert k.run("clamp", (x, torch.zeros(1, device="cuda"), None)) is None   # bound not 0-d
    assert k.run("silu", (x.cpu(),)) is None                             # device
    empty = torch.empty(0, 8, device="cuda")
    out = k.run("bias_relu", (empty, torch.zeros(8, device="cuda")))
    assert out.shape == (0, 8)
    first, second = k.run("swiglu_backward", (empty, empty, empty))
    assert first.shape == second.shape == (0, 8)
    enable_fused_kernels(False)
    try:
        assert try_fused("silu", x) is None
    finally:
        enable_fused_kernels(True)
    _close(try_fused("silu", x), A.silu(x.cpu().numpy()))
