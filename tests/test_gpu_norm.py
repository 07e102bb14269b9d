"""GPU parity of the RMS / layer normalization kernels (nt_norm_forward / nt_norm_backward).

float32 results within 2e-6 of each array's largest magnitude (sums in other orders;
rsqrtf within 2 ulp of 1/sqrt); float16 / bfloat16 outputs within one unit of the stored type.
"""
import numpy as np
import pytest
import torch

from conftest import REPO
from namitorch_b200.backends import enable_fused_kernels, get_backend, try_fused_normalization
from oracle import normalization as O
from oracle.casts import round_to_bf16

pytestmark = pytest.mark.gpu
GOLDEN = np.load(REPO / "tests" / "golden" / "norm.npz")
TORCH = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _store(x, dt):
    if dt == "bf16":
        return round_to_bf16(np.asarray(x, np.float32))
    if dt == "f16":
        return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)
    return np.asarray(x, np.float32)


def _close(got, want, dt="f32", rel=2e-6, rows=1):
    got = got.float().cpu().numpy() if isinstance(got, torch.Tensor) else got
    scale = float(np.max(np.abs(want))) if want.size else 0.0
    if dt == "f32":
        assert float(np.max(np.abs(got - want), initial=0.0)) <= rel * max(scale, 1e-30) * max(1, rows) ** 0.5
    else:
        ulp = 2.0 ** (-7 if dt == "bf16" else -10)
        np.testing.assert_allclose(got, want, rtol=ulp, atol=ulp * scale * 1e-2 + 1e-6)


def _k():
    return get_backend(torch.zeros(1, device="cuda")).normalization


def test_reference_golden_cases(cuda_device):
    d = GOLDEN
    t = {k: torch.from_numpy(d[k]).cuda() for k in d.files}
    y, st = _k().run("layer_norm", (t["layer_x"], t["layer_w"], t["layer_b"]), eps=1e-5)
    _close(y, d["layer_y"], rel=4e-6)
    dx, dw, db = _k().run("layer_norm_backward", (t["layer_x"], t["layer_w"], t["layer_g"], st))
    _close(dx, d["layer_dx"], rel=4e-6)
    _close(dw, d["layer_dw"], rel=4e-6, rows=60)
    _close(db, d["layer_db"], rel=4e-6, rows=60)
    y, st = _k().run("rms_norm", (t["rms_x"], t["rms_w"], None), eps=1e-6)
    _close(y, d["rms_y"], rel=4e-6)
    dx, dw, db = _k().run("rms_norm_backward", (t["rms_x"], t["rms_w"], t["rms_g"], st), needs=(True, True, False))
    assert db is None
    _close(dx, d["rms_dx"], rel=4e-6)
    _close(dw, d["rms_dw"], rel=4e-6, rows=35)


WIDTHS = [1, 7, 8, 33, 64, 100, 256, 768, 1000, 1024, 2048, 3000, 4096, 5000, 8192]


@pytest.mark.parametrize("dt", list(TORCH))
@pytest.mark.parametrize("width", WIDTHS)
@pytest.mark.parametrize("layer", [True, False], ids=["layer", "rms"])
def test_widths_dtypes_match_oracle(cuda_device, dt, width, layer):
    rng = np.random.default_rng(width + 7 * layer)
    rows = 37
    x = _store((rng.normal(0, 1.5, (rows, width)) + 2).astype(np.float32), dt)
    w = _store(rng.normal(1, 0.3, width).astype(np.float32), dt)
    b = _store(rng.normal(0, 0.3, width).astype(np.float32), dt) if layer else None
    g = _store(rng.normal(0, 1, (rows, width)).astype(np.float32), dt)
    cu = lambda a: None if a is None else torch.from_numpy(a).cuda().to(TORCH[dt])
    name = "layer_norm" if layer else "rms_norm"
    y, st = _k().run(name, (cu(x), cu(w), cu(b)), eps=1e-5)
    want_y, want_st = O.forward(x, w, b, 1e-5, layer)
    np.testing.assert_allclose(st.cpu().numpy(), want_st, rtol=2e-6, atol=2e-6)
    _close(y, want_y, dt)
    dx, dw, db = _k().run(name + "_backward", (cu(x), cu(w), cu(g), st))
    st_ours = st.cpu().numpy()
    want_dx, want_dw, want_db = O.backward(x, w, g, st_ours, layer)
    _close(dx, want_dx, dt, rel=4e-6)
    _close(dw, _store(want_dw, dt), dt, rel=4e-6, rows=rows)
    _close(db, _store(want_db, dt), dt, rel=4e-6, rows=rows)


def test_without_affine_zero_rows_and_declines(cuda_device):
    x = torch.randn(4, 64, device="cuda")
    y, st = _k().run("layer_norm", (x, None, None), eps=1e-5, save_stats=False)
    assert st is None
    want, _ = O.forward(x.cpu().numpy(), None, None, 1e-5, True)
    _close(y, want)
    empty = torch.zeros(0, 64, device="cuda")
    y, st = _k().run("rms_norm", (empty, None, None), eps=1e-5)
    assert y.shape == (0, 64) and st.shape == (0, 2)
    dx, dw, db = _k().run("rms_norm_backward", (empty, torch.ones(64, device="cuda"), empty, st))
    assert dx.shape == (0, 64) and torch.all(dw == 0) and torch.all(db == 0)
    assert _k().run("layer_norm", (torch.zeros(2, 9000, device="cuda"), None, None), eps=1e-5) is None
    assert _k().run("rms_norm", (x, None, torch.zeros(64, device="cuda")), eps=1e-5) is None   # no bias for RMS
    assert _k().run("layer_norm", (x.double(), None, None), eps=1e-5) is None
    with pytest.raises(ValueError, match="positive and finite"):
        _k().run("layer_norm", (x, None, None), eps=0.0)
    with pytest.raises(TypeError, match="three Python bools"):
        _k().run("layer_norm_backward", (x, None, x, torch.zeros(4, 2, device="cuda")), needs=(True, 1, True))
    enable_fused_kernels(False)
    try:
        assert try_fused_normalization("layer_norm", x, None, None, eps=1e-5) is None
    finally:
        enable_fused_kernels(True)
    assert try_fused_normalization("layer_norm", x, None, None, eps=1e-5) is not None


@pytest.mark.parametrize("rows,width,dt,layer,needs", [
    (20000, 64, "f32", True, (True, True, True)),       # four rows per block, many rows per block
    (3001, 999, "f32", True, (False, True, True)),      # per-element path, affine sums only
    (2500, 2048, "f16", False, (False, True, False)),   # weight gradient alone
    (1500, 5000, "bf16", True, (True, False, True)),    # bias gradient with the input gradient
])
def test_many_rows_affine_sums_match_oracle_and_repeat(cuda_device, rows, width, dt, layer, needs):
    rng = np.random.default_rng(rows + width)
    x = _store((rng.normal(0, 1.5, (rows, width)) + 2).astype(np.float32), dt)
    w = _store(rng.normal(1, 0.3, width).astype(np.float32), dt)
    b = _store(rng.normal(0, 0.3, width).astype(np.float32), dt) if layer else None
    g = _store(rng.normal(0, 1, (rows, width)).astype(np.float32), dt)
    tx, tw, tg = (torch.from_numpy(a).cuda().to(TORCH[dt]) for a in (x, w, g))
    tb = torch.from_numpy(b).cuda().to(TORCH[dt]) if layer else None
    op = "layer_norm" if layer else "rms_norm"
    _, st = _k().run(op, (tx, tw, tb), eps=1e-5)
    _, want_st = O.forward(x, w, b, 1e-5, layer)
    want_dx, want_dw, want_db = O.backward(x, w, g, want_st, layer)
    first = _k().run(op + "_backward", (tx, tw, tg, st), needs=needs)
    second = _k().run(op + "_backward", (tx, tw, tg, st), needs=needs)
    for got, again, want, need in zip(first, second, (want_dx, want_dw, want_db), needs):
        if not need:
            assert got is None
            continue
        assert torch.equal(got, again)                   # a fixed summation order
    if needs[0]:
        _close(first[0], _store(want_dx, dt), dt, rel=4e-6)
    if needs[1]:
        _close(first[1], _store(want_dw, dt), dt, rel=4e-6, rows=rows)
    if needs[2]:
        _close(first[2], _store(want_db, dt), dt, rel=4e-6, rows=rows)
