"""The optimizer tail captured as a CUDA graph (namitorch_b200.training.CapturedOptimizerStep)
against the same loop run eagerly: identical master weights, moments, model copy, step
counts, loss scale, growth tracker and learning-rate counter, bit for bit, over iterations
with overflowing gradients (skipped steps), scale growth and a device-gated schedule. The
eager side is itself checked against the oracle in test_gpu_schedule.py.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import to_params
from namitorch_b200 import GradScaler
from namitorch_b200 import workloads as W
from namitorch_b200.optim import AdamW, WarmupCosine, clip_grad_norm_
from namitorch_b200.training import CapturedOptimizerStep
from oracle.casts import round_to_bf16

pytestmark = pytest.mark.gpu

STEPS = 14
OVERFLOW = {3, 7, 8}
CONFIG = {"warmup_steps": 3, "total_steps": 12, "min_lr": 1e-5}


def _grads(shape, step):
    grads = [round_to_bf16(g * np.float32(512.0)) for g in W.outlier_grads(shape, seed=70 + step)]
    if step in OVERFLOW:
        grads[5].reshape(-1)[11] = np.inf
    return grads


def _setup(shape, arrays, staged, dtype):
    params = to_params(arrays)
    decay, no_decay = shape.groups()
    opt = AdamW([{"params": [params[i] for i in decay], "lr": 1e-3, "weight_decay": 0.1},
                 {"params": [params[i] for i in no_decay], "lr": 3e-4, "weight_decay": 0.0}],
                lr=1e-3, betas=(0.9, 0.999), eps=1e-8, model_dtype=dtype)
    sched = WarmupCosine(opt, **CONFIG)
    scaler = GradScaler(init_scale=512.0, growth_interval=2)
    for p, g in zip(params, staged[0]):
        p.grad = g.clone()
    return params, opt, sched, scaler


def _state(params, opt, sched, scaler):
    eng = opt._engine
    torch.cuda.synchronize()
    return {"master": eng.master.cpu().numpy(), "m": eng.exp_avg.cpu().numpy(), "v": eng.exp_avg_sq.cpu().numpy(),
            "copy": eng.copy.view(torch.int16).cpu().numpy(), "steps": eng.steps.cpu().numpy(),
            "scale": scaler.get_scale(), "tracker": int(scaler._tracker_dev.item()),
            "last_step": sched.last_step, "lrs": [v.hex() for v in sched.get_last_lr()]}


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_replays_match_the_eager_loop_bit_for_bit(cuda_device, dtype):
    shape = W.CONFIG_SMALL
    arrays = W.init_params(shape, seed=4)
    staged = [[torch.from_numpy(g).to("cuda", dtype) for g in _grads(shape, s)] for s in range(STEPS)]
    one = torch.ones((), device="cuda")

    # Eager loop.
    params, opt, sched, scaler = _setup(shape, arrays, staged, dtype)
    norms_eager = []
    for step in range(STEPS):
        for p, g in zip(params, staged[step]):
            p.grad.copy_(g)
        scaler.scale(one)
        scaler.unscale_(opt)
        norms_eager.append(clip_grad_norm_(params, 1.0).clone())
        updated = scaler.step(opt)
        scaler.update()
        sched.step(updated)
    eager = _state(params, opt, sched, scaler)

    # One eager iteration, then graph replays of the same tail.
    params, opt, sched, scaler = _setup(shape, arrays, staged, dtype)
    norms_graph = []
    for step in range(STEPS):
        for p, g in zip(params, staged[step]):
            p.grad.copy_(g)
        scaler.scale(one)
        if step == 0:
            scaler.unscale_(opt)
            norms_graph.append(clip_grad_norm_(params, 1.0).clone())
            updated = scaler.step(opt)
            scaler.update()
            sched.step(updated)
            captured = CapturedOptimizerStep(opt, scaler, params, max_norm=1.0, scheduler=sched, capacity=64)
            continue
        captured()
        norms_graph.append(captured.norm.clone())
    graph = _state(params, opt, sched, scaler)

    assert captured.replays == STEPS - 1
    for key in ("master", "m", "v", "copy", "steps"):
        assert np.array_equal(graph[key], eager[key]), key
    for key in ("scale", "tracker", "last_step", "lrs"):
        assert graph[key] == eager[key], key
    assert graph["last_step"] == STEPS - len(OVERFLOW)
    assert torch.equal(torch.stack(norms_graph), torch.stack(norms_eager))
    # The host view (the groups' "lr") reads the device counter the replays advanced.
    assert [g["lr"] for g in opt.param_groups] == [float.fromhex(h) for h in eager["lrs"]]


@pytest.mark.filterwarnings("ignore:The CUDA Graph is empty")   # the refused step leaves nothing captured
def test_capture_requires_an_eager_step_and_bounds_replays(cuda_device):
    shape = W.CONFIG_SMALL
    arrays = W.init_params(shape, seed=5)
    params = to_params(arrays)
    opt = AdamW(params, lr=1e-3, model_dtype=torch.bfloat16)
    scaler = GradScaler(init_scale=256.0)
    for p in params:
        p.grad = torch.zeros(p.shape, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="eager"):
        CapturedOptimizerStep(opt, scaler, params, max_norm=1.0)
    scaler.scale(torch.ones((), device="cuda"))
    scaler.step(opt)
    scaler.update()
    step = CapturedOptimizerStep(opt, scaler, params, max_norm=1.0, capacity=2)
    step()
    step()
    with pytest.raises(RuntimeError, match="sized for 2 replays"):
        step()
    with pytest.raises(RuntimeError, match="not allowed during CUDA graph capture"):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            opt.step()
