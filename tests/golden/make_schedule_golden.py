"""Generates ``schedules.json`` by running the reference's learning-rate schedulers.

For every scheduler class of namitorch/optim/lr_scheduler.py, a reference AdamW with two
parameter groups (base lrs 1e-3 and 3e-4) is built, the scheduler constructed (some with a
nonzero last_step) and stepped 40 times; the groups' lr after construction and after every
step is recorded as float.hex, with the final state_dict.

Usage (needs the reference checkout; not run by the tests):
    python tests/golden/make_schedule_golden.py /path/to/reference
"""
from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

CASES = [
    ("StepLR", {"step_size": 7, "gamma": 0.5}, 0),
    ("MultiStepLR", {"milestones": [5, 17, 30], "gamma": 0.3}, 0),
    ("ExponentialLR", {"gamma": 0.93}, 3),
    ("CosineAnnealingLR", {"T_max": 25, "eta_min": 1e-5}, 0),
    ("LinearLR", {"start_factor": 0.25, "end_factor": 1.0, "total_iters": 12}, 0),
    ("WarmupCosine", {"warmup_steps": 6, "total_steps": 30, "min_lr": 1e-5}, 0),
    ("WarmupCosine", {"warmup_steps": 0, "total_steps": 9, "min_lr": 0.0}, 2),
]


def main(reference: str) -> None:
    sys.path.insert(0, reference)
    import namitorch as nt
    from namitorch import optim
    from namitorch.nn import Parameter
    out = []
    for name, config, last_step in CASES:
        a = Parameter(nt.tensor(np.zeros(3, np.float32)))
        b = Parameter(nt.tensor(np.zeros(2, np.float32)))
        opt = optim.AdamW([{"params": [a], "lr": 1e-3}, {"params": [b], "lr": 3e-4, "weight_decay": 0.0}],
                          lr=1e-3, weight_decay=0.1, fused=False)
        cls = getattr(optim.lr_scheduler, name)
        sched = cls(opt, **config, last_step=last_step)
        seq = [[float(g["lr"]).hex() for g in opt.param_groups]]
        for _ in range(40):
            sched.step()
            seq.append([float(g["lr"]).hex() for g in opt.param_groups])
        sd = sched.state_dict()
        out.append({"name": name, "config": config, "last_step": last_step, "lrs": seq,
                    "state": {k: (v if not isinstance(v, float) else v.hex()) for k, v in sd.items()
                              if k != "base_lrs"}, "base_lrs": [float(x).hex() for x in sd["base_lrs"]]})
    (HERE / "schedules.json").write_text(json.dumps(out, indent=1) + "\n")
    print("wrote schedules.json")


if __name__ == "__main__":
    main(sys.argv[1])
