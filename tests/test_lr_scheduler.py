"""Learning-rate schedulers on the host path, against the reference's own sequences.

``tests/golden/schedules.json`` holds the lr of both parameter groups after construction
and after each of 40 steps for every scheduler class of the reference, with its final
state_dict (``tests/golden/make_schedule_golden.py``). The host path and the oracle must
reproduce every value bit for bit.
"""
import json

import pytest
import torch

from conftest import REPO
from namitorch_b200.optim import Optimizer, lr_scheduler
from oracle import lr_schedule as O

CASES = json.loads((REPO / "tests" / "golden" / "schedules.json").read_text())


def _optimizer():
    a = torch.nn.Parameter(torch.zeros(3))
    b = torch.nn.Parameter(torch.zeros(2))
    return Optimizer([{"params": [a], "lr": 1e-3, "weight_decay": 0.1},
                      {"params": [b], "lr": 3e-4, "weight_decay": 0.0}], {"lr": 1e-3})


@pytest.mark.parametrize("case", CASES, ids=[f"{c['name']}-{i}" for i, c in enumerate(CASES)])
def test_host_schedule_matches_reference_bit_for_bit(case):
    opt = _optimizer()
    cls = getattr(lr_scheduler, case["name"])
    sched = cls(opt, **case["config"], last_step=case["last_step"])
    seq = [[float(g["lr"]).hex() for g in opt.param_groups]]
    for _ in range(40):
        sched.step()
        seq.append([float(g["lr"]).hex() for g in opt.param_groups])
    assert seq == case["lrs"]
    sd = sched.state_dict()
    assert sd["last_step"] == case["state"]["last_step"] and sd["scheduler"] == case["name"]
    assert sd["config"] == case["state"]["config"] and [v.hex() for v in sd["base_lrs"]] == case["base_lrs"]


@pytest.mark.parametrize("case", CASES, ids=[f"{c['name']}-{i}" for i, c in enumerate(CASES)])
def test_oracle_schedule_matches_reference(case):
    bases = [1e-3, 3e-4]
    for k, want in enumerate(case["lrs"]):
        got = O.lrs(case["name"], case["last_step"] + k, bases, case["config"])
        assert [v.hex() for v in got] == want


def test_gate_and_state_round_trip():
    opt = _optimizer()
    sched = lr_scheduler.WarmupCosine(opt, warmup_steps=3, total_steps=10)
    sched.step(False)
    assert sched.last_step == 0
    sched.step(True)
    assert sched.last_step == 1
    state = sched.state_dict()
    other = lr_scheduler.WarmupCosine(_optimizer(), warmup_steps=3, total_steps=10)
    other.load_state_dict(state)
    assert other.last_step == 1 and other.get_last_lr() == sched.get_last_lr()


def test_validation_follows_reference():
    with pytest.raises(ValueError, match="warmup_steps must be smaller"):
        lr_scheduler.WarmupCosine(_optimizer(), warmup_steps=5, total_steps=5)
    with pytest.raises(ValueError, match="Minimum learning rate"):
        lr_scheduler.CosineAnnealingLR(_optimizer(), T_max=3, eta_min=1.0)
    with pytest.raises(TypeError, match="step_size must be an integer"):
        lr_scheduler.StepLR(_optimizer(), step_size=1.5)
    with pytest.raises(TypeError, match="milestones"):
        lr_scheduler.MultiStepLR(_optimizer(), milestones={1, 2})
    with pytest.raises(TypeError, match="NamiTorch Optimizer"):
        lr_scheduler.StepLR(object(), step_size=1)
