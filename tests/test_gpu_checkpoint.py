"""Resuming from the reference's own checkpoint on the GPU.

``tests/golden/checkpoint_ref.zip`` holds the reference's AdamW (three NumPy steps) and
GradScaler state; the reference then took a fourth step whose parameter checksums are in
``checkpoint_expect.json``. Loaded into this package's AdamW, the same fourth step must
give the same bytes, the re-exported optimizer entry must be the reference's (same archive
metadata, same arrays), and a checkpoint written here must load back into a fresh optimizer.
"""
import hashlib
import json

import numpy as np
import pytest
import torch

from conftest import REPO
from namitorch_b200 import GradScaler
from namitorch_b200 import checkpoint as C
from namitorch_b200.optim import AdamW

pytestmark = pytest.mark.gpu
GOLDEN = REPO / "tests" / "golden"
EXPECT = json.loads((GOLDEN / "checkpoint_expect.json").read_text())
NAMES = EXPECT["names"]
SHAPES = [tuple(s) for s in EXPECT["shapes"]]
GROUP_NAMES = [["a.weight", "b.weight"], ["a.bias", "b.bias"]]


def grads_for(step: int) -> list[np.ndarray]:
    """The fixture script's gradients for `step` (same seeds and distribution)."""
    rng = np.random.default_rng(EXPECT["grad_seed_base"] + step)
    return [rng.normal(0.0, 0.05, s).astype(np.float32) for s in SHAPES]


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(np.ascontiguousarray(t.detach().cpu().numpy()).tobytes()).hexdigest()


def build(model_state, fused=None):
    params = {n: torch.nn.Parameter(model_state[n].detach().clone().cuda()) for n in NAMES}
    opt = AdamW([{"params": [params[n] for n in GROUP_NAMES[0]], "weight_decay": 0.1},
                 {"params": [params[n] for n in GROUP_NAMES[1]], "weight_decay": 0.0}],
                lr=1e-2, betas=(0.9, 0.999), eps=1e-8, fused=fused)
    return params, opt


def test_resume_reference_checkpoint_matches_reference_fourth_step(cuda_device, tmp_path):
    ck = C.load(GOLDEN / "checkpoint_ref.zip")
    params, opt = build(ck["model"])
    scaler = GradScaler()
    info = C.load_checkpoint(GOLDEN / "checkpoint_ref.zip", opt, scaler, parameter_names=GROUP_NAMES)
    assert info["step"] == 3 and info["cumulative_tokens"] == 12345
    assert scaler.get_scale() == 512.0 and scaler.state_dict()["growth_tracker"] == 0
    # The optimizer entry this package exports is the reference's, node for node.
    ours, ours_arrays = C.metadata_bytes(C.pack_optimizer(opt))
    ref, ref_arrays = C.metadata_bytes(ck["optimizer"])
    assert ours == ref
    for (_, a), (_, b) in zip(ours_arrays, ref_arrays):
        assert a.dtype == b.dtype and np.array_equal(a, b)
    # The fourth step reproduces the reference's bytes.
    for n, g in zip(NAMES, grads_for(EXPECT["next_step"])):
        params[n].grad = torch.from_numpy(g).cuda()
    opt.step()
    for n in NAMES:
        assert sha(params[n]) == EXPECT["after_step4_sha"][n], n
    # A checkpoint written here loads back into a fresh optimizer with the same state.
    out = tmp_path / "ours.zip"
    C.save_checkpoint(out, opt, scaler, model_state={n: params[n].detach() for n in NAMES},
                      parameter_names=GROUP_NAMES, step=4, epoch=1, cumulative_tokens=12345 + 4)
    params2, opt2 = build(C.load(out)["model"])
    scaler2 = GradScaler()
    info2 = C.load_checkpoint(out, opt2, scaler2, parameter_names=GROUP_NAMES)
    assert info2["step"] == 4 and scaler2.get_scale() == 512.0
    a, b = opt.state_dict(), opt2.state_dict()
    assert a["param_groups"] == b["param_groups"]
    for k in a["state"]:
        assert a["state"][k]["step"] == b["state"][k]["step"] == 4
        for name in ("exp_avg", "exp_avg_sq"):
            assert torch.equal(a["state"][k][name].cpu(), b["state"][k][name].cpu())


def test_reference_state_into_the_multi_tensor_path(cuda_device):
    """The reference's state (saved with fused=False) drives the fused multi-tensor kernel
    after the groups are switched back to fused=None: same fourth step."""
    ck = C.load(GOLDEN / "checkpoint_ref.zip")
    params, opt = build(ck["model"])
    state = C.unpack_optimizer(ck["optimizer"])
    for group in state["param_groups"]:
        group["fused"] = None
    state["defaults"]["fused"] = None
    opt.load_state_dict(state)
    for n, g in zip(NAMES, grads_for(EXPECT["next_step"])):
        params[n].grad = torch.from_numpy(g).cuda()
    opt.step()
    assert opt._uses_engine()
    for n in NAMES:
        assert sha(params[n]) == EXPECT["after_step4_sha"][n], n
