"""Helpers shared by the GPU parity tests (torch <-> NumPy plumbing, checksums)."""
import hashlib

import numpy as np
import torch

from namitorch_b200 import workloads as W


def sha(*arrays) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def to_params(arrays, device="cuda"):
    return [torch.nn.Parameter(torch.from_numpy(np.ascontiguousarray(a)).to(device)) for a in arrays]


def set_grads(params, grads, dtype=None):
    for p, g in zip(params, grads):
        if g is None:
            p.grad = None
            continue
        t = torch.from_numpy(np.ascontiguousarray(g)).to(p.device)
        p.grad = t.to(dtype if dtype is not None else p.dtype)


def groups(shape: W.GPTShape, params, weight_decay=W.ADAMW_OPTIONS["weight_decay"]):
    decay, no_decay = shape.groups()
    return [{"params": [params[i] for i in decay], "weight_decay": weight_decay},
            {"params": [params[i] for i in no_decay], "weight_decay": 0.0}]


def state_numpy(opt, params):
    """(master params, exp_avg list, exp_avg_sq list, steps) in parameter order, via state_dict."""
    sd = opt.state_dict()
    order = {id(p): i for i, p in enumerate(params)}
    registered = opt._registered_parameters()
    idx_of = {k: order[id(p)] for k, p in enumerate(registered)}
    n = len(params)
    ps, ms, vs, steps = [None] * n, [None] * n, [None] * n, [0] * n
    for k, st in sd["state"].items():
        i = idx_of[k]
        ms[i] = st["exp_avg"].cpu().numpy()
        vs[i] = st["exp_avg_sq"].cpu().numpy()
        steps[i] = st["step"]
        if "master_param" in st:
            ps[i] = st["master_param"].cpu().numpy()
    for i, p in enumerate(params):
        if ps[i] is None:
            ps[i] = p.detach().float().cpu().numpy() if p.dtype == torch.float32 else None
    if any(p is None for p in ps):
        masters = opt.master_params
        order_reg = {id(p): k for k, p in enumerate(registered)}
        for i, p in enumerate(params):
            if ps[i] is None:
                ps[i] = masters[order_reg[id(p)]].cpu().numpy()
    return ps, ms, vs, steps


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
