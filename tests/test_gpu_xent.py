"""GPU parity of the fused softmax cross-entropy against the reference fixtures and the oracle.

Bar: loss within 1e-5 relative; dlogits within one bfloat16 ulp (bf16 logits) of the
reference / oracle gradient rounded to bfloat16, float32 gradients within 1e-5 relative."""
import numpy as np
import pytest
import torch

from conftest import GOLDEN, load_golden
from namitorch_b200 import workloads as W
from namitorch_b200.nn.functional import cross_entropy, softmax_cross_entropy
from oracle import xent as oxent
from oracle.casts import bf16_bits_to_f32, f32_to_bf16_bits, round_to_bf16

pytestmark = pytest.mark.gpu


def bf16_ulp_distance(a_bits: np.ndarray, b_bits: np.ndarray) -> np.ndarray:
    """Distance in bfloat16 units in the last place between two bit-pattern arrays."""
    def ordered(bits):
        b = bits.astype(np.int32)
        return np.where(b & 0x8000, 0x8000 - (b & 0x7FFF), 0x8000 + b)
    return np.abs(ordered(a_bits) - ordered(b_bits))


def to_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


def assert_bf16_close(ours: torch.Tensor, ref_f32: np.ndarray, max_ulp: int = 1, abs_tol: float = 0.0):
    """Within ``max_ulp`` bfloat16 ulps of the reference rounded to bfloat16, or within ``abs_tol``.

    ``abs_tol`` covers label smoothing, where p*a - eps/V cancels: both implementations
    evaluate exp(x - lse) in float32 with ~6e-7 relative error, so near cancellation
    the bound scales with the operand eps/(V*D), not with the tiny result."""
    ours_bits = to_bits(ours).reshape(-1)
    d = bf16_ulp_distance(ours_bits, f32_to_bf16_bits(ref_f32).reshape(-1))
    if abs_tol:
        diff = np.abs(bf16_bits_to_f32(ours_bits) - np.asarray(ref_f32, np.float32).reshape(-1))
        d = np.where(diff <= abs_tol, 0, d)
    assert int(d.max()) <= max_ulp, f"max bf16 ulp distance {int(d.max())}"


def smoothing_tol(eps: float, classes: int, denominator: float, max_weight: float = 1.0) -> float:
    return 1e-5 * eps * max_weight / (classes * denominator)


CASES = {
    "cfg4_64rows_mean": ({}, lambda t: t),
    "cfg4_64rows_ignore": ({}, lambda t: np.where(np.arange(t.size) % 5 == 0, -100, t)),
    "cfg4_64rows_weight_smooth": ({"weight": True, "label_smoothing": 0.1},
                                  lambda t: np.where(np.arange(t.size) % 5 == 0, -100, t)),
    "cfg4_64rows_sum": ({"reduction": "sum"}, lambda t: t),
    "cfg4_64rows_smooth": ({"label_smoothing": 0.2}, lambda t: t),
}


@pytest.mark.parametrize("name", list(CASES))
def test_config4_rows_match_reference(cuda_device, name):
    gold = load_golden("xent.json")["cases"][name]
    arrays = np.load(GOLDEN / "xent_arrays.npz")
    kw, tfn = CASES[name]
    logits, targets = W.xent_inputs(rows=64, classes=W.XENT_CLASSES, seed=0)
    targets = tfn(targets)
    x = torch.from_numpy(logits).cuda().to(torch.bfloat16)
    t = torch.from_numpy(targets).cuda()
    kwargs = dict(kw)
    if kwargs.pop("weight", False):
        kwargs["weight"] = torch.from_numpy(arrays["cfg4_weight"]).cuda()
    loss, dl = softmax_cross_entropy(x, t, **kwargs)
    ref = float.fromhex(gold["loss_hex"][0])
    assert abs(float(loss.item()) - ref) <= 1e-5 * abs(ref)
    cols = arrays["cols"]
    eps = kwargs.get("label_smoothing", 0.0)
    valid = int((targets != -100).sum())
    wmax = float(arrays["cfg4_weight"].max()) if "weight" in kwargs else 1.0
    den = valid if kwargs.get("reduction", "mean") == "mean" else 1.0
    if "weight" in kwargs:
        den = float(arrays["cfg4_weight"][targets[targets != -100]].sum())
    tol = smoothing_tol(eps, W.XENT_CLASSES, den, wmax) if eps else 0.0
    assert_bf16_close(dl[:, torch.from_numpy(cols).cuda()], arrays[name + "__grad_cols"], abs_tol=tol)
    tgt = torch.from_numpy(np.clip(targets, 0, None)).cuda()
    assert_bf16_close(dl[torch.arange(64, device="cuda"), tgt], arrays[name + "__grad_target"], abs_tol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("classes", [1, 7, 8, 100, 4097, 50257])
@pytest.mark.parametrize("reduction", ["mean", "sum", "none"])
def test_shapes_dtypes_reductions_match_oracle(cuda_device, dtype, classes, reduction):
    rng = np.random.default_rng(classes)
    rows = 37
    x32 = rng.normal(0, 2, (rows, classes)).astype(np.float32)
    if dtype is torch.bfloat16:
        x32 = round_to_bf16(x32)
    elif dtype is torch.float16:
        x32 = x32.astype(np.float16).astype(np.float32)
    targets = rng.integers(0, classes, rows)
    targets[3] = -100
    loss, dl = softmax_cross_entropy(torch.from_numpy(x32).cuda().to(dtype), torch.from_numpy(targets).cuda(),
                                     reduction=reduction)
    ref_loss, ref_dl = oxent.cross_entropy(x32, targets, reduction=reduction)
    np.testing.assert_allclose(np.atleast_1d(loss.cpu().numpy()), np.atleast_1d(ref_loss), rtol=1e-5, atol=1e-6)
    if dtype is torch.bfloat16:
        assert_bf16_close(dl, ref_dl)
    elif dtype is torch.float16:
        np.testing.assert_allclose(dl.float().cpu().numpy(), ref_dl, rtol=2e-3, atol=2e-7)
    else:
        np.testing.assert_allclose(dl.cpu().numpy(), ref_dl, rtol=1e-5, atol=1e-9)


def test_weights_and_smoothing_match_oracle(cuda_device):
    rng = np.random.default_rng(1)
    x = round_to_bf16(rng.normal(0, 2, (50, 1000)).astype(np.float32))
    t = rng.integers(0, 1000, 50)
    t[::7] = -1
    w = rng.uniform(0.2, 2.0, 1000).astype(np.float32)
    for eps in (0.0, 0.1):
        loss, dl = softmax_cross_entropy(torch.from_numpy(x).cuda().to(torch.bfloat16), torch.from_numpy(t).cuda(),
                                         weight=torch.from_numpy(w).cuda(), ignore_index=-1, label_smoothing=eps)
        rl, rdl = oxent.cross_entropy(x, t, weight=w, ignore_index=-1, label_smoothing=eps)
        assert abs(float(loss.item()) - float(rl)) <= 1e-5 * abs(float(rl))
        den = float(w[t[t != -1]].sum())
        assert_bf16_close(dl, rdl, abs_tol=smoothing_tol(eps, 1000, den, float(w.max())) if eps else 0.0)


def test_edge_rows_match_reference(cuda_device):
    gold = load_golden("xent.json")["cases"]
    arrays = np.load(GOLDEN / "xent_arrays.npz")
    x = torch.from_numpy(arrays["edge_logits"]).cuda()
    t = torch.from_numpy(arrays["small_targets"]).cuda()
    loss, dl = softmax_cross_entropy(x, t)
    ref = float.fromhex(gold["edge_mean"]["loss_hex"][0])
    assert np.isnan(ref) == np.isnan(float(loss.item()))
    np.testing.assert_allclose(dl.cpu().numpy(), arrays["edge_mean__grad"], rtol=1e-5, atol=1e-8, equal_nan=True)
    loss, dl = softmax_cross_entropy(torch.from_numpy(arrays["small_logits"]).cuda(), torch.full((6,), -100).cuda())
    assert float(loss.item()) == 0.0 and float(dl.abs().sum().item()) == 0.0


def test_bad_target_raises_index_error(cuda_device):
    x = torch.zeros(4, 10, device="cuda")
    with pytest.raises(IndexError):
        softmax_cross_entropy(x, torch.tensor([0, 10, 1, 2], device="cuda"))


def test_autograd_backward_scales_by_upstream(cuda_device):
    rng = np.random.default_rng(2)
    x32 = round_to_bf16(rng.normal(0, 2, (16, 3000)).astype(np.float32))
    t = torch.from_numpy(rng.integers(0, 3000, 16)).cuda()
    x = torch.from_numpy(x32).cuda().to(torch.bfloat16).requires_grad_()
    loss = cross_entropy(x, t)
    (loss * 1024.0).backward()
    _, rdl = oxent.cross_entropy(x32, t.cpu().numpy())
    assert_bf16_close(x.grad, rdl * np.float32(1024.0))
    x2 = torch.from_numpy(x32).cuda().requires_grad_()
    per_row = cross_entropy(x2.view(4, 4, 3000), t.view(4, 4), reduction="none")
    assert per_row.shape == (4, 4)
    up = torch.arange(16, dtype=torch.float32, device="cuda").view(4, 4)
    per_row.backward(up)
    _, rdl_none = oxent.cross_entropy(x32, t.cpu().numpy(), reduction="none")
    np.testing.assert_allclose(x2.grad.cpu().numpy(), rdl_none * np.arange(16, dtype=np.float32)[:, None],
                               rtol=1e-5, atol=1e-9)


def test_full_config4_properties(cuda_device):
    """[8192, 50257] bf16: per-row results on a sample of rows match the oracle; every
    gradient row sums to ~0 (softmax minus one-hot); the mean loss matches the row losses."""
    logits, targets = W.xent_inputs(seed=0)
    x = torch.from_numpy(logits).cuda().to(torch.bfloat16)
    t = torch.from_numpy(targets).cuda()
    loss, dl = softmax_cross_entropy(x, t)
    rows = np.random.default_rng(0).choice(W.XENT_ROWS, 64, replace=False)
    xs = bf16_bits_to_f32(to_bits(x[torch.from_numpy(rows).cuda()]))
    per_row, _ = oxent.cross_entropy(xs, targets[rows], reduction="none", with_grad=False)
    loss_none, dl_none = softmax_cross_entropy(x[torch.from_numpy(rows).cuda()], t[torch.from_numpy(rows).cuda()],
                                               reduction="none")
    np.testing.assert_allclose(loss_none.cpu().numpy(), per_row, rtol=1e-5)
    _, ref_dl = oxent.cross_entropy(xs, targets[rows])
    assert_bf16_close(dl[torch.from_numpy(rows).cuda()] * 8192 / 64, ref_dl, max_ulp=2)
    sums = dl.float().sum(dim=1).abs().max().item()
    assert sums < 1e-6
    assert np.isfinite(float(loss.item())) and 10.0 < float(loss.item()) < 14.0


@pytest.mark.parametrize("dtype,rows,classes,shift", [
    (torch.float32, 1500, 1000, 0),      # several rows per block: chunk refills with the next row
    (torch.bfloat16, 3000, 4097, 0),     # rows start at every 2-byte offset within 16 bytes
    (torch.float16, 2000, 333, 0),       # rows shorter than a chunk's share of the threads
    (torch.bfloat16, 700, 999, 1),       # logits not 16-byte aligned: the unstaged passes
])
def test_many_rows_and_unaligned_match_oracle(cuda_device, dtype, rows, classes, shift):
    rng = np.random.default_rng(rows + classes)
    x32 = rng.normal(0, 2, (rows, classes)).astype(np.float32)
    if dtype is torch.bfloat16:
        x32 = round_to_bf16(x32)
    elif dtype is torch.float16:
        x32 = x32.astype(np.float16).astype(np.float32)
    targets = rng.integers(0, classes, rows)
    targets[::11] = -100
    flat = torch.empty(rows * classes + shift, dtype=dtype, device="cuda")
    x = flat[shift:].view(rows, classes)
    x.copy_(torch.from_numpy(x32).to(dtype))
    assert (x.data_ptr() % 16 == 0) == (shift == 0)
    loss, dl = softmax_cross_entropy(x, torch.from_numpy(targets).cuda())
    ref_loss, ref_dl = oxent.cross_entropy(x32, targets)
    assert abs(float(loss.item()) - float(ref_loss)) <= 1e-5 * abs(float(ref_loss))
    if dtype is torch.bfloat16:
        assert_bf16_close(dl, ref_dl)
    elif dtype is torch.float16:
        np.testing.assert_allclose(dl.float().cpu().numpy(), ref_dl, rtol=2e-3, atol=2e-7)
    else:
        np.testing.assert_allclose(dl.cpu().numpy(), ref_dl, rtol=1e-5, atol=1e-9)


@pytest.mark.parametrize("shift", [0, 1])
def test_forward_only_writes_no_gradient(cuda_device, shift):
    """Logits that do not require grad: the launch has no dlogits; the loss still matches."""
    rng = np.random.default_rng(9 + shift)
    rows, classes = 600, 2049
    x32 = round_to_bf16(rng.normal(0, 2, (rows, classes)).astype(np.float32))
    t = rng.integers(0, classes, rows)
    flat = torch.empty(rows * classes + shift, dtype=torch.bfloat16, device="cuda")
    x = flat[shift:].view(rows, classes)
    x.copy_(torch.from_numpy(x32).to(torch.bfloat16))
    loss = cross_entropy(x, torch.from_numpy(t).cuda())
    assert loss.grad_fn is None
    ref_loss, _ = oxent.cross_entropy(x32, t, with_grad=False)
    assert abs(float(loss.item()) - float(ref_loss)) <= 1e-5 * abs(float(ref_loss))


def test_rows_wider_than_the_shared_memory_buffer(cuda_device):
    """150000 bf16 classes (300 KB rows) exceed one CTA's shared memory: the passes read
    global memory instead of a staged row."""
    rng = np.random.default_rng(21)
    rows, classes = 24, 150_000
    x32 = round_to_bf16(rng.normal(0, 2, (rows, classes)).astype(np.float32))
    t = rng.integers(0, classes, rows)
    t[5] = -100
    loss, dl = softmax_cross_entropy(torch.from_numpy(x32).cuda().to(torch.bfloat16), torch.from_numpy(t).cuda())
    ref_loss, ref_dl = oxent.cross_entropy(x32, t)
    assert abs(float(loss.item()) - float(ref_loss)) <= 1e-5 * abs(float(ref_loss))
    assert_bf16_close(dl, ref_dl)
