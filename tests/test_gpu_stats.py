"""GPU parity of the gradient-statistics, clipping and loss-scale kernels against the oracle."""
import math

import numpy as np
import pytest
import torch

from gpu_helpers import to_params
from namitorch_b200 import GradScaler
from namitorch_b200 import _native as N
from namitorch_b200.flat import grad_stats_for
from namitorch_b200.optim import clip_grad_norm_, clip_grad_value_, get_grad_norm
from oracle import amp as oamp
from oracle import clip as oclip
from oracle.casts import round_to_bf16

pytestmark = pytest.mark.gpu
NORM = N.STATS_FIELDS.index("norm")
FOUND = N.STATS_FIELDS.index("found_inf")


def _grads(dtype, seed=0, sizes=(1, 5, 8, 1000, 8191, 8192, 8193, 100003)):
    rng = np.random.default_rng(seed)
    out = []
    for n in sizes:
        g = rng.normal(0, 1e-2, n).astype(np.float32)
        g[rng.random(n) < 0.01] *= 100
        if dtype is torch.bfloat16:
            g = round_to_bf16(g)
        elif dtype is torch.float16:
            g = g.astype(np.float16).astype(np.float32)
        out.append(g)
    return out


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("p", [2.0, float("inf"), 1.0, 3.5])
def test_norm_matches_oracle(cuda_device, dtype, p):
    grads = _grads(dtype)
    tensors = [torch.from_numpy(g).cuda().to(dtype) for g in grads]
    stats = grad_stats_for(tensors, norm_type=p)
    ref = float(oclip.total_norm(grads, p))
    ours = float(stats[NORM].item())
    assert abs(ours - ref) <= 1e-12 * ref
    assert stats[FOUND].item() == 0.0


def test_nonfinite_norms_follow_reference(cuda_device):
    for values, expect in (([1.0, np.nan, 2.0], "nan"), ([1.0, np.inf, -3.0], "inf"), ([-np.inf, 0.5], "inf"),
                           ([0.0, 0.0], 0.0)):
        g = torch.tensor(values, dtype=torch.float32, device="cuda")
        stats = grad_stats_for([g])
        norm = float(stats[NORM].item())
        ref = float(oclip.total_norm([np.asarray(values, np.float32)]))
        if expect == "nan":
            assert math.isnan(norm) and math.isnan(ref)
        else:
            assert norm == ref
        assert stats[FOUND].item() == (0.0 if expect == 0.0 else 1.0)


def test_empty_gradient_list(cuda_device):
    stats = grad_stats_for([], device=torch.device("cuda", 0))
    assert stats[NORM].item() == 0.0 and stats[FOUND].item() == 0.0


def test_unscaled_found_inf_and_overflow(cuda_device):
    """found_inf is taken on g / scale: finite scaled values can overflow when the scale is < 1."""
    g = torch.tensor([3e38, 1.0], dtype=torch.float32, device="cuda")
    scale = torch.tensor([0.5], dtype=torch.float32, device="cuda")
    assert grad_stats_for([g], scale=scale)[FOUND].item() == 1.0
    assert grad_stats_for([g], scale=torch.tensor([4.0], device="cuda"))[FOUND].item() == 0.0


def test_clip_on_plain_tensors_rewrites_like_reference(cuda_device):
    grads = _grads(torch.float32, seed=3)
    params = to_params([np.zeros_like(g) for g in grads])
    for p, g in zip(params, grads):
        p.grad = torch.from_numpy(g).cuda()
    ref = [g.copy() for g in grads]
    ref_norm = oclip.clip_grad_norm_(ref, 0.5)
    norm = clip_grad_norm_(params, 0.5)
    assert abs(float(norm.item()) - float(ref_norm)) <= 1e-12 * float(ref_norm)
    for p, r in zip(params, ref):
        np.testing.assert_allclose(p.grad.cpu().numpy(), r, rtol=2e-7, atol=0)
    with pytest.raises(RuntimeError, match="nonfinite"):
        params[0].grad[0] = float("nan")
        clip_grad_norm_(params, 0.5, error_if_nonfinite=True)


def test_get_grad_norm_and_clip_value(cuda_device):
    grads = _grads(torch.bfloat16, seed=4)
    params = to_params([np.zeros_like(g) for g in grads])
    for p, g in zip(params, grads):
        p.grad = torch.from_numpy(g).cuda()
    assert abs(float(get_grad_norm(params, 1.0).item()) - float(oclip.total_norm(grads, 1.0))) <= 1e-12 * float(
        oclip.total_norm(grads, 1.0))
    clip_grad_value_(params, 0.05)
    ref = [g.copy() for g in grads]
    oclip.clip_grad_value_(ref, 0.05)
    for p, r in zip(params, ref):
        np.testing.assert_array_equal(p.grad.cpu().numpy(), r)


@pytest.mark.parametrize("growth,backoff,interval,init", [(2.0, 0.5, 3, 65536.0), (3.0, 0.25, 2, 1e-30),
                                                           (10.0, 0.9, 1, 3e38), (1.5, 0.125, 4, 7.0)])
def test_scaler_update_trajectory_bit_exact(cuda_device, growth, backoff, interval, init):
    rng = np.random.default_rng(int(growth * 10))
    pattern = rng.random(40) < 0.3
    scaler = GradScaler(init, growth, backoff, interval)
    oscaler = oamp.OracleGradScaler(init, growth, backoff, interval)
    p = torch.nn.Parameter(torch.zeros(4, device="cuda"))

    class _Opt:
        param_groups = [{"params": [p]}]

        def _parameters_with_grad(self):
            yield self.param_groups[0], p, p.grad

        def _amp_unscale_(self, scale, lazy):
            return grad_stats_for([p.grad], scale=scale)

        def _amp_enable_skip(self):
            pass

        def step(self):
            pass

    opt = _Opt()
    for inject in pattern:
        p.grad = torch.tensor([1.0, 2.0, float("inf") if inject else 3.0, 4.0], device="cuda")
        scaler.scale(torch.ones((), device="cuda"))
        scaler.step(opt)
        scaler.update()
        oscaler.update(bool(inject))
        assert float(scaler.get_scale()).hex() == float(oscaler.scale).hex()
        assert scaler.state_dict()["growth_tracker"] == oscaler.growth_tracker


def test_scaler_state_dict_roundtrip(cuda_device):
    s = GradScaler(1024.0, 2.0, 0.5, 5)
    s.scale(torch.ones((), device="cuda"))
    s._optimizer_states.clear()
    s._scale_used = False
    d = s.state_dict()
    t = GradScaler()
    t.load_state_dict(d)
    assert t.state_dict() == d
    with pytest.raises(ValueError):
        t.load_state_dict({**d, "growth_tracker": 99})


def _as_dtype(x: np.ndarray, dtype) -> np.ndarray:
    if dtype is torch.bfloat16:
        return round_to_bf16(x)
    if dtype is torch.float16:
        return x.astype(np.float16).astype(np.float32)
    return x.astype(np.float32)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("scale", [None, 1024.0, 3.0])
@pytest.mark.parametrize("poison", [False, True])
def test_stats_on_misaligned_spans_match_oracle(cuda_device, dtype, scale, poison):
    """Gradients as views at odd element offsets of one buffer: every chunk starts off a
    16-byte boundary (the staged kernel masks the first vector and reads the elements after
    the last boundary with plain loads). With `poison`, a NaN sits in a masked head vector
    and an inf in a plain-load tail."""
    rng = np.random.default_rng(5)
    sizes = [1, 3, 7, 8, 9, 15, 17, 8191, 8192, 8193, 16385, 50001]
    offsets, off = [], 1
    for n in sizes:
        offsets.append(off)
        off += n + 3
    flat = _as_dtype(rng.normal(0, 1, off + 8).astype(np.float32) * np.float32(scale or 1.0), dtype)
    if poison:
        flat[offsets[9]] = np.nan                    # first element of an unaligned span
        flat[offsets[10] + sizes[10] - 1] = np.inf   # last element of another
    buf = torch.from_numpy(flat).cuda().to(dtype)
    views = [buf[o:o + n] for o, n in zip(offsets, sizes)]
    arrays = [flat[o:o + n].copy() for o, n in zip(offsets, sizes)]
    scale_t = None if scale is None else torch.tensor([scale], dtype=torch.float32, device="cuda")
    stats = grad_stats_for(views, scale=scale_t)
    s = dict(zip(N.STATS_FIELDS, stats.cpu().numpy()))
    unscaled = [a if scale is None else a / np.float32(scale) for a in arrays]
    if poison:
        assert s["nonfinite"] == 2 and s["nan"] == 1 and s["found_inf"] == 1.0 and math.isnan(s["norm"])
        return
    ref = float(oclip.total_norm(unscaled, 2.0))
    assert abs(s["norm"] - ref) <= 1e-12 * ref
    assert s["maxabs"] == max(float(np.max(np.abs(u))) for u in unscaled)
    assert s["found_inf"] == 0.0 and s["error"] == 0.0


@pytest.mark.parametrize("dtype,values,scale", [
    # f32(g / 0.25) overflows for g = 2^126: found_inf, as the reference's float32 unscale.
    (torch.bfloat16, [1.0, 2.0 ** 126, -3.0], 0.25),
    (torch.float32, [1.0, 2.0 ** 126, -3.0], 0.25),
    # Below-overflow neighbour: stays finite.
    (torch.bfloat16, [1.0, 2.0 ** 125, -3.0], 0.25),
    # fp16 with a tiny scale (2^-20): the bit-level pass declines it (2^(1008+20) is not a
    # double); the conversion path gives the same answer.
    (torch.float16, [1.0, 60000.0, -2.0 ** -24], 2.0 ** -20),
    # Exact zeros and subnormals of every format.
    (torch.bfloat16, [0.0, -0.0, 2.0 ** -133, 1e-3, 0.0], 1.0),
    (torch.float16, [0.0, 2.0 ** -24, -2.0 ** -20, 0.5], 65536.0),
    (torch.float32, [0.0, 2.0 ** -149, -2.0 ** -130, 7.0], 1.0),
])
def test_pow2_scale_edges_match_reference_unscale(cuda_device, dtype, values, scale):
    g = np.asarray(values, np.float32)
    t = torch.from_numpy(g).cuda().to(dtype)
    stored = t.float().cpu().numpy()
    stats = grad_stats_for([t], scale=torch.tensor([scale], dtype=torch.float32, device="cuda"))
    s = dict(zip(N.STATS_FIELDS, stats.cpu().numpy()))
    with np.errstate(over="ignore"):
        u = stored / np.float32(scale)   # the reference's float32 unscale
    finite = np.isfinite(u)
    assert s["nonfinite"] == np.count_nonzero(~finite)
    assert s["found_inf"] == (0.0 if finite.all() else 1.0)
    if finite.all():
        ref = float(oclip.total_norm([u], 2.0))
        assert abs(s["norm"] - ref) <= 1e-12 * ref
        assert s["maxabs"] == float(np.max(np.abs(u)))
    else:
        assert s["norm"] == np.inf
