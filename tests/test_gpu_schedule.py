"""The training loop's optimizer tail with no host synchronisation, against the oracle.

``scaler.unscale_ -> clip_grad_norm_ -> scaler.step -> scaler.update -> scheduler.step(gate)``
(namitorch/training/runner.py:247-254 with ``if updated: scheduler.step()`` made a device
decision). Gradients overflow on some steps, so the scheduler must hold still exactly on
the skipped steps. The steady-state iterations run under torch's synchronisation debug
mode set to "error": any host read of device state would raise.
"""
import numpy as np
import pytest
import torch

from gpu_helpers import state_numpy, to_params
from namitorch_b200 import GradScaler
from namitorch_b200 import workloads as W
from namitorch_b200.optim import AdamW, WarmupCosine
from namitorch_b200.optim import clip_grad_norm_
from oracle import adamw as oadamw
from oracle import amp as oamp
from oracle import lr_schedule as O
from oracle.casts import round_to_bf16

pytestmark = pytest.mark.gpu

STEPS = 12
OVERFLOW = {2, 5, 6}          # steps whose gradients hold an inf
CONFIG = {"warmup_steps": 3, "total_steps": 10, "min_lr": 1e-5}
BASES = [1e-3, 3e-4]


def _grads(shape, step, scale):
    grads = [round_to_bf16(g * np.float32(scale)) for g in W.normal_grads(shape, seed=50 + step)]
    if step in OVERFLOW:
        grads[3].reshape(-1)[7] = np.inf
    return grads


def test_device_gated_schedule_matches_oracle_without_host_syncs(cuda_device):
    shape = W.CONFIG_SMALL
    arrays = W.init_params(shape, seed=3)
    params = to_params(arrays)
    decay, no_decay = shape.groups()
    opt = AdamW([{"params": [params[i] for i in decay], "lr": BASES[0], "weight_decay": 0.1},
                 {"params": [params[i] for i in no_decay], "lr": BASES[1], "weight_decay": 0.0}],
                lr=BASES[0], betas=(0.9, 0.999), eps=1e-8, model_dtype=torch.bfloat16)
    sched = WarmupCosine(opt, **CONFIG)
    scaler = GradScaler(init_scale=1024.0, growth_interval=4)
    one = torch.ones((), device="cuda")
    # Every step's scaled bf16 gradients are staged on the device beforehand (the scale each
    # step uses is known from the oracle's trajectory below).
    oscaler = oamp.OracleGradScaler(1024.0, 2.0, 0.5, 4)
    scales, stepped = [], []
    for step in range(STEPS):
        scales.append(oscaler.scale)
        finite = step not in OVERFLOW
        stepped.append(finite)
        oscaler.update(not finite)
    staged = [[torch.from_numpy(g).to("cuda", torch.bfloat16) for g in _grads(shape, s, scales[s])]
              for s in range(STEPS)]
    for p, g in zip(params, staged[0]):
        p.grad = g.clone()

    def iteration(step):
        for p, g in zip(params, staged[step]):
            p.grad.copy_(g)
        scaler.scale(one)
        scaler.unscale_(opt)
        clip_grad_norm_(params, 1.0)
        updated = scaler.step(opt)
        scaler.update()
        sched.step(updated)

    for step in range(2):   # warm-up: segment tables and the schedule table are built here
        iteration(step)
    torch.cuda.synchronize()
    torch.cuda.set_sync_debug_mode("error")
    try:
        for step in range(2, STEPS):
            iteration(step)
    finally:
        torch.cuda.set_sync_debug_mode("default")
    torch.cuda.synchronize()

    # Oracle: the same loop on the host, the scheduler stepped only after applied steps.
    oracle = oadamw.OracleAdamW([a.copy() for a in arrays],
                                [(decay, {"lr": BASES[0], "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay": 0.1}),
                                 (no_decay, {"lr": BASES[1], "betas": (0.9, 0.999), "eps": 1e-8,
                                             "weight_decay": 0.0})])
    oscaler = oamp.OracleGradScaler(1024.0, 2.0, 0.5, 4)
    used, final_step = O.gated_lrs("WarmupCosine", BASES, CONFIG, stepped)
    for step in range(STEPS):
        for (indices, options), lr in zip(oracle.groups, used[step]):
            options["lr"] = lr
        r = oamp.amp_step(oracle, oscaler, [g.astype(np.float32) for g in _grads(shape, step, scales[step])],
                          max_norm=1.0)
        assert r["stepped"] == stepped[step]
    assert sched.last_step == final_step == STEPS - len(OVERFLOW)
    want = O.lrs("WarmupCosine", final_step, BASES, CONFIG)
    assert [v.hex() for v in sched.get_last_lr()] == [v.hex() for v in want]
    assert [g["lr"] for g in opt.param_groups] == want
    assert scaler.get_scale() == oscaler.scale
    # The clip coefficient comes from this package's one-pass norm (within 1e-12 of the
    # reference's two-pass norm), so the states agree to float32 rounding, not bit for bit.
    ps, ms, vs, steps = state_numpy(opt, params)
    for i in range(len(arrays)):
        np.testing.assert_allclose(ps[i], oracle.params[i], rtol=1e-6, atol=1e-9)
        np.testing.assert_allclose(ms[i], oracle.state[i]["exp_avg"], rtol=1e-6, atol=1e-12)
        assert steps[i] == oracle.state[i]["step"]


def test_gated_schedule_refuses_the_per_tensor_path(cuda_device):
    p = torch.nn.Parameter(torch.zeros(16, device="cuda"))
    opt = AdamW([p], lr=1e-3, fused=False)
    sched = WarmupCosine(opt, warmup_steps=1, total_steps=4)
    scaler = GradScaler()
    p.grad = torch.ones(16, device="cuda")
    scaler.scale(torch.ones((), device="cuda"))
    updated = scaler.step(opt)
    scaler.update()
    sched.step(updated)
    p.grad = torch.ones(16, device="cuda")
    with pytest.raises(RuntimeError, match="multi-tensor path"):
        opt.step()
