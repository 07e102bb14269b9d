"""GPU parity of the row-softmax kernels (nt_row_softmax) with the reference and the oracle.

Tolerances: float32 outputs within 1e-5 relative of the oracle (exp on the SFU and a
reciprocal of the row sum, each a few float32 ulps from expf / IEEE division; sum orders
differ); float16 / bfloat16 outputs within one unit of the stored type.
"""
import numpy as np
import pytest
import torch

from conftest import REPO
from namitorch_b200.backends import enable_fused_kernels, get_backend, try_fused_softmax
from oracle import softmax as S
from oracle.casts import round_to_bf16

pytestmark = pytest.mark.gpu
GOLDEN = np.load(REPO / "tests" / "golden" / "softmax.npz")
TORCH = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def _store(x: np.ndarray, dt: str) -> np.ndarray:
    """float32 -> storage type -> float32 (the values a kernel of that dtype reads and writes)."""
    if dt == "bf16":
        return round_to_bf16(x)
    if dt == "f16":
        return x.astype(np.float16).astype(np.float32)
    return x.astype(np.float32)


def _run(op, *arrays, **kw):
    out = get_backend(arrays[0]).softmax.run(op, arrays, **kw)
    assert out is not None, "the kernel declined supported arrays"
    torch.cuda.synchronize()
    return out


def _check(got, want, dt, rtol=1e-5, atol=1e-7):
    got = got.float().cpu().numpy()
    if dt == "f32":
        np.testing.assert_allclose(got, want, rtol=rtol, atol=atol)
    else:
        ulp = 2.0 ** (-7 if dt == "bf16" else -10)
        np.testing.assert_allclose(got, want, rtol=ulp, atol=atol)


# causal_poisoned: NaN and +inf in the blocked positions, which the reference ignores (the
# forward never reads whole blocked vectors).
@pytest.mark.parametrize("name", ["plain", "masked", "causal", "causal_poisoned"])
def test_reference_golden_cases(cuda_device, name):
    x = torch.from_numpy(GOLDEN[f"{name}_x"]).cuda()
    g = torch.from_numpy(GOLDEN[f"{name}_g"]).cuda()
    if name == "plain":
        y = _run("softmax", x)
        dx = _run("softmax_backward", y, g)
    elif name == "masked":
        mask = torch.from_numpy(GOLDEN["masked_mask"]).cuda()
        y = _run("masked_softmax", x, mask, require_nonempty=True)
        dx = _run("masked_softmax_backward", y, g, mask)
    else:
        kw = {"query_position_offset": int(GOLDEN["causal_offset"])}
        y = _run("causal_softmax", x, None, require_nonempty=True, **kw)
        dx = _run("causal_softmax_backward", y, g, None, **kw)
    _check(y, GOLDEN[f"{name}_y"], "f32")
    _check(dx, GOLDEN[f"{name}_dx"], "f32", atol=1e-6)


WIDTHS = [1, 7, 8, 64, 100, 256, 257, 1000, 1024, 1025, 2000, 2048, 3000, 4096]


@pytest.mark.parametrize("dt", list(TORCH))
@pytest.mark.parametrize("width", WIDTHS)
def test_width_buckets_and_paths_match_oracle(cuda_device, dt, width):
    rng = np.random.default_rng(width)
    shape = (3, 5, width)
    x = _store(rng.normal(0, 3, shape).astype(np.float32), dt)
    g = _store(rng.normal(0, 1, shape).astype(np.float32), dt)
    mask = rng.random((5, width)) < 0.6
    mask[:, 0] = True
    xt, gt = torch.from_numpy(x).cuda().to(TORCH[dt]), torch.from_numpy(g).cuda().to(TORCH[dt])
    mt = torch.from_numpy(mask).cuda()
    for op, extra, kw, okw in (("softmax", (), {}, {}),
                               ("masked_softmax", (mt,), {}, {"mask": mask}),
                               ("causal_softmax", (None,), {"query_position_offset": 1}, {"causal": True, "offset": 1})):
        y = _run(op, xt, *extra, **kw)
        want, _ = S.forward(x, **okw)
        _check(y, want, dt)
        ys = _store(y.float().cpu().numpy(), dt)
        dx = _run(op + "_backward", y, gt, *extra, **kw)
        _check(dx, S.backward(ys, g, **okw), dt, atol=1e-6)


def test_empty_and_invalid_rows_follow_reference(cuda_device):
    x = torch.tensor([[1.0, 2.0, 3.0, 4.0], [-np.inf] * 4, [1.0, float("nan"), 0.0, 2.0], [float("inf"), 0, 1, 2]],
                     device="cuda")
    y = _run("softmax", x)
    want, status = S.forward(x.cpu().numpy())
    got = y.cpu().numpy()
    np.testing.assert_allclose(got[0], want[0], rtol=1e-6)
    assert np.all(got[1] == 0) and np.all(np.isnan(got[2])) and np.all(np.isnan(got[3]))
    with pytest.raises(ValueError, match="finite or -inf"):
        get_backend(x).softmax.run("masked_softmax", (x, torch.ones(4, dtype=torch.bool, device="cuda")),
                                   require_nonempty=True)
    mask = torch.tensor([True, True, False, False], device="cuda")
    scores = torch.zeros(2, 3, 4, device="cuda")
    scores[1, 2, :2] = -float("inf")
    with pytest.raises(ValueError, match=r"Attention row \(1, 2\) has no allowed keys"):
        get_backend(scores).softmax.run("masked_softmax", (scores, mask), require_nonempty=True)


def test_seam_declines_and_switch(cuda_device):
    k = get_backend(torch.zeros(1, device="cuda")).softmax
    assert k.run("softmax", (torch.zeros(4, 5000, device="cuda"),)) is None          # wider than 4096
    assert k.run("softmax", (torch.zeros(4, 8, dtype=torch.float64, device="cuda"),)) is None
    assert k.run("causal_softmax", (torch.zeros(8, device="cuda"), None)) is None      # causal needs 2-D
    assert k.run("masked_softmax", (torch.zeros(2, 8, device="cuda"),
                                    torch.ones(3, 8, dtype=torch.bool, device="cuda"))) is None
    assert k.run("softmax", (torch.zeros(0, 8, device="cuda"),)).shape == (0, 8)
    enable_fused_kernels(False)
    try:
        assert try_fused_softmax("softmax", torch.zeros(2, 8, device="cuda")) is None
    finally:
        enable_fused_kernels(True)
    assert try_fused_softmax("softmax", torch.zeros(2, 8, device="cuda")) is not None


def test_attention_sized_causal_rows_are_distributions(cuda_device):
    """[8*12*1024, 1024] bf16 causal scores (GPT-2 small attention): every row sums to one on
    its allowed prefix and is zero past the diagonal."""
    gen = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(8 * 12, 1024, 1024, device="cuda", generator=gen).to(torch.bfloat16)
    y = _run("causal_softmax", x, None, require_nonempty=True).float()
    sums = y.sum(-1)
    assert torch.allclose(sums, torch.ones_like(sums), atol=2e-2)
    upper = torch.triu(torch.ones(1024, 1024, dtype=torch.bool, device="cuda"), diagonal=1)
    assert not torch.any(y[:, upper])


@pytest.mark.parametrize("dt", list(TORCH))
@pytest.mark.parametrize("width,offset", [(64, 0), (1024, 0), (1024, 37), (4096, 5)])
def test_causal_forward_ignores_the_masked_part(cuda_device, dt, width, offset):
    """The causal forward never uses scores past the diagonal (the reference's rule: a
    disallowed column enters as -inf). NaN and +inf planted there leave every row as the
    oracle computes it; vectors wholly past the diagonal are not read at all."""
    rng = np.random.default_rng(width + offset)
    queries = 24
    x = _store(rng.normal(0, 3, (2, queries, width)).astype(np.float32), dt)
    for q in range(queries):
        lo = offset + q + 1
        if lo < width:
            x[:, q, lo:] = np.where(rng.random((2, width - lo)) < 0.5, np.nan, np.inf)
    xt = torch.from_numpy(x).cuda().to(TORCH[dt])
    y = _run("causal_softmax", xt, None, query_position_offset=offset)
    want, _ = S.forward(x, causal=True, offset=offset)
    assert not np.isnan(want).any()
    _check(y, want, dt)
