"""Learning-rate schedules on the host path, against the reference's own sequences.

``tests/golden/schedules.json`` holds the lr of both parameter groups after construction
and after each of 40 steps for every scheduler class of the reference, with its final
state_dict (``tests/golden/make_schedule_golden.py``). WarmupCosine (built in) must
reproduce its sequences bit for bit; every other reference scheduler runs through the
generic ``Schedule`` with the oracle's restatement of its formula as ``lr_at``, which
exercises the same stepping, state and table machinery. The oracle must match every case.
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
    if case["name"] == "WarmupCosine":
        sched = lr_scheduler.WarmupCosine(opt, **case["config"], last_step=case["last_step"])
    else:
        def lr_at(step, base, name=case["name"], config=case["config"]):
            return O.lrs(name, step, [base], config)[0]
        sched = lr_scheduler.Schedule(opt, lr_at, last_step=case["last_step"], name=case["name"],
                                      config=case["config"])
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
        lr_scheduler.WarmupCosine(_optimizer(), warmup_steps=1, total_steps=3, min_lr=1.0)
    with pytest.raises(TypeError, match="warmup_steps must be an integer"):
        lr_scheduler.WarmupCosine(_optimizer(), warmup_steps=1.5, total_steps=3)
    with pytest.raises(ValueError, match="total_steps must be at least 1"):
        lr_scheduler.WarmupCosine(_optimizer(), warmup_steps=0, total_steps=0)
    with pytest.raises(ValueError, match="min_lr must be finite and nonnegative"):
        lr_scheduler.WarmupCosine(_optimizer(), warmup_steps=0, total_steps=2, min_lr=-1.0)
    with pytest.raises(TypeError, match="NamiTorch Optimizer"):
        lr_scheduler.WarmupCosine(object(), warmup_steps=0, total_steps=2)
    with pytest.raises(TypeError, match="lr_at must be a callable"):
        lr_scheduler.Schedule(_optimizer(), 0.5)


def test_state_loads_only_into_the_same_schedule():
    sched = lr_scheduler.WarmupCosine(_optimizer(), warmup_steps=2, total_steps=9)
    sched.step()
    state = sched.state_dict()
    other = lr_scheduler.Schedule(_optimizer(), lambda step, base: base)
    with pytest.raises(ValueError, match="does not match"):
        other.load_state_dict(state)
    bad = dict(state, config={"warmup_steps": 9, "total_steps": 9, "min_lr": 0.0})
    target = lr_scheduler.WarmupCosine(_optimizer(), warmup_steps=2, total_steps=9)
    with pytest.raises(ValueError, match="warmup_steps must be smaller"):
        target.load_state_dict(bad)
    assert target.config == {"warmup_steps": 2, "total_steps": 9, "min_lr": 0.0} and target.last_step == 0
    target.load_state_dict(state)
    assert target.last_step == 1 and target.get_last_lr() == sched.get_last_lr()
