"""Generates the golden fixtures in this directory by running the reference itself.

The reference (renderityai/NamiTorch) is pure Python over NumPy, so its CPU path imports
and runs in the development container. This script drives its public API —
``namitorch.optim.AdamW`` (fused=False, the NumPy path), ``namitorch.amp.GradScaler``,
``namitorch.optim.clip_grad_norm_`` / ``get_grad_norm`` and
``namitorch.nn.functional.cross_entropy`` with autograd — on the seeded inputs of
``namitorch_b200.workloads`` and records SHA-256 checksums of the resulting float32 /
float16 / bfloat16 bytes, scalar results (as float.hex) and small sampled arrays.

Usage (needs the reference checkout; not run by the tests):
    python tests/golden/make_golden.py /path/to/reference [--full]
``--full`` adds the 124M-parameter configuration-2 run (a few minutes, ~4 GB of RAM).
"""
from __future__ import annotations

import argparse
import os
import hashlib
import json
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from namitorch_b200 import workloads as W  # noqa: E402
from oracle.casts import f32_to_bf16_bits, round_to_bf16  # noqa: E402


def sha(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def load_reference(path: str):
    sys.path.insert(0, path)
    import namitorch as nt  # noqa: F401
    from namitorch import amp as nt_amp
    from namitorch import optim as nt_optim
    from namitorch.nn import Parameter
    from namitorch.nn import functional as F
    return nt, nt_optim, nt_amp, Parameter, F


def make_params(nt, Parameter, arrays):
    return [Parameter(nt.tensor(a.copy())) for a in arrays]


def groups_for(shape: W.GPTShape, params, weight_decay: float):
    decay, no_decay = shape.groups()
    return [{"params": [params[i] for i in decay], "weight_decay": weight_decay},
            {"params": [params[i] for i in no_decay], "weight_decay": 0.0}]


def set_grads(nt, params, grads):
    for p, g in zip(params, grads):
        p._grad = None if g is None else nt.tensor(np.ascontiguousarray(g, dtype=np.float32))


def state_arrays(opt, params):
    out = []
    for p in params:
        st = opt.state.get(id(p), {})
        out.append((np.asarray(p._data), np.asarray(st["exp_avg"]._data) if "exp_avg" in st else None,
                    np.asarray(st["exp_avg_sq"]._data) if "exp_avg_sq" in st else None, st.get("step", 0)))
    return out


def summarize_state(opt, params, copy_dtype: str | None = None) -> dict:
    arrays = state_arrays(opt, params)
    ps = [a[0] for a in arrays]
    ms = [a[1] for a in arrays if a[1] is not None]
    vs = [a[2] for a in arrays if a[2] is not None]
    out = {
        "sha256_param": sha(*ps),
        "sha256_exp_avg": sha(*ms),
        "sha256_exp_avg_sq": sha(*vs),
        "param_steps": [a[3] for a in arrays],
        "per_tensor_sha256_param": [sha(p) for p in ps],
        "head_param": [[float(x).hex() for x in p.reshape(-1)[:4]] for p in ps[:4]],
    }
    if copy_dtype == "f16":
        out["sha256_copy_f16"] = sha(*[p.astype(np.float16) for p in ps])
    if copy_dtype == "bf16":
        out["sha256_copy_bf16"] = sha(*[f32_to_bf16_bits(p) for p in ps])
    return out


def adamw_config0(ref) -> dict:
    nt, nt_optim, _, Parameter, _ = ref
    shape = W.CONFIG_SMALL
    params = make_params(nt, Parameter, W.init_params(shape, seed=0))
    opt = nt_optim.AdamW(groups_for(shape, params, W.ADAMW_OPTIONS["weight_decay"]), lr=W.ADAMW_OPTIONS["lr"],
                         betas=W.ADAMW_OPTIONS["betas"], eps=W.ADAMW_OPTIONS["eps"], fused=False)
    grads = W.normal_grads(shape, seed=0)
    t0 = time.perf_counter()
    for _ in range(10):
        set_grads(nt, params, grads)
        opt.step()
    seconds = time.perf_counter() - t0
    out = {"config": "0", "shape": shape.name, "steps": 10, "options": W.ADAMW_OPTIONS,
           "grad_seed": 0, "param_seed": 0, "reference_seconds": seconds}
    out.update(summarize_state(opt, params))
    return out


def adamw_variants(ref) -> dict:
    """Small explicit cases: maximize, lr = 0, Adam (coupled decay), subnormal / huge values."""
    nt, nt_optim, _, Parameter, _ = ref
    rng = np.random.default_rng(7)
    cases = {}
    base_p = rng.normal(0, 1, (3, 37)).astype(np.float32)
    base_g = rng.normal(0, 1e-2, (3, 37)).astype(np.float32)
    base_p[0, :4] = [1e-40, -3e-39, 1e30, -0.0]
    base_g[0, :4] = [1e-41, 2e-38, -1e20, 0.0]
    variants = {
        "adamw_default": dict(cls="AdamW", lr=1e-3, weight_decay=1e-2, maximize=False),
        "adamw_maximize": dict(cls="AdamW", lr=1e-2, weight_decay=0.5, maximize=True),
        "adamw_lr0": dict(cls="AdamW", lr=0.0, weight_decay=0.1, maximize=False),
        "adamw_wd0": dict(cls="AdamW", lr=5e-3, weight_decay=0.0, maximize=False),
        "adam_coupled": dict(cls="Adam", lr=1e-3, weight_decay=0.05, maximize=False),
        "adam_betas": dict(cls="AdamW", lr=2e-3, weight_decay=0.01, maximize=False, betas=(0.5, 0.75), eps=1e-3),
    }
    for name, v in variants.items():
        p = Parameter(nt.tensor(base_p.copy()))
        kwargs = dict(lr=v["lr"], weight_decay=v["weight_decay"], maximize=v["maximize"],
                      betas=v.get("betas", (0.9, 0.999)), eps=v.get("eps", 1e-8))
        if v["cls"] == "AdamW":
            kwargs["fused"] = False
        opt = getattr(nt_optim, v["cls"])([p], **kwargs)
        for k in range(5):
            p._grad = nt.tensor((base_g * (k + 1)).astype(np.float32))
            opt.step()
        st = opt.state[id(p)]
        cases[name] = {
            "options": {**kwargs, "cls": v["cls"]},
            "param": np.asarray(p._data).view(np.uint32).reshape(-1).tolist(),
            "exp_avg": np.asarray(st["exp_avg"]._data).view(np.uint32).reshape(-1).tolist(),
            "exp_avg_sq": np.asarray(st["exp_avg_sq"]._data).view(np.uint32).reshape(-1).tolist(),
            "step": st["step"],
        }
    return {"param_seed": 7, "shape": [3, 37], "steps": 5, "grad_rule": "base_g * (k+1)",
            "base_param": base_p.view(np.uint32).reshape(-1).tolist(),
            "base_grad": base_g.view(np.uint32).reshape(-1).tolist(), "cases": cases}


def amp_config1(ref) -> dict:
    nt, nt_optim, nt_amp, Parameter, _ = ref
    shape = W.CONFIG_SMALL
    params = make_params(nt, Parameter, W.init_params(shape, seed=0))
    opt = nt_optim.AdamW(groups_for(shape, params, W.ADAMW_OPTIONS["weight_decay"]), lr=W.ADAMW_OPTIONS["lr"],
                         betas=W.ADAMW_OPTIONS["betas"], eps=W.ADAMW_OPTIONS["eps"], fused=False)
    scaler = nt_amp.GradScaler(init_scale=65536.0, growth_factor=2.0, backoff_factor=0.5, growth_interval=4)
    inf_idx = W.inf_positions(int(np.prod(shape.shapes()[0][1])), 0.001, seed=0)
    trace = []
    for step in range(12):
        scale = scaler.get_scale()
        base = W.normal_grads(shape, seed=1000 + step)
        g16 = [(g * np.float32(scale)).astype(np.float16) for g in base]
        if step == 3:
            flat = g16[0].reshape(-1)
            flat[inf_idx] = np.float16(np.inf)
        set_grads(nt, params, [g.astype(np.float32) for g in g16])
        scaler.scale(nt.tensor(np.float32(1.0)))
        finite = scaler.unscale_(opt)
        stepped = scaler.step(opt)
        scaler.update()
        trace.append({"scale_used": float(scale).hex(), "finite": bool(finite), "stepped": bool(stepped),
                      "scale_after": float(scaler.get_scale()).hex(),
                      "growth_tracker": scaler.state_dict()["growth_tracker"]})
    out = {"config": "1", "shape": shape.name, "steps": 12, "options": W.ADAMW_OPTIONS,
           "scaler": {"init_scale": 65536.0, "growth_factor": 2.0, "backoff_factor": 0.5, "growth_interval": 4},
           "grad_rule": "f16(normal_grads(seed=1000+step) * scale_used); step 3: tok_emb[inf_positions(seed=0)] = +inf",
           "inf_count": int(inf_idx.size), "trace": trace}
    out.update(summarize_state(opt, params, copy_dtype="f16"))
    return out


def clip_cases(ref) -> dict:
    nt, nt_optim, _, Parameter, _ = ref
    shape = W.CONFIG_SMALL
    cases = {}
    base = [round_to_bf16(g) for g in W.outlier_grads(shape, seed=2)]
    for name, grads, p, max_norm in [
        ("bf16_outliers_p2", base, 2.0, 1.0),
        ("bf16_outliers_pinf", base, float("inf"), 1.0),
        ("bf16_outliers_p1", base, 1.0, 5.0),
        ("bf16_outliers_p3.5", base, 3.5, 0.25),
        ("small_noclip_p2", [g * np.float32(1e-3) for g in base], 2.0, 1.0),
        ("zeros_p2", [np.zeros_like(g) for g in base[:3]], 2.0, 1.0),
    ]:
        params = make_params(nt, Parameter, [np.zeros_like(g) for g in grads])
        set_grads(nt, params, grads)
        norm = nt_optim.clip_grad_norm_(params, max_norm, norm_type=p)
        clipped = [np.asarray(q.grad._data) for q in params]
        cases[name] = {"norm_type": p, "max_norm": max_norm, "norm": float(np.asarray(norm._data)).hex(),
                       "sha256_clipped": sha(*clipped), "n_tensors": len(grads)}
    specials = {}
    for name, values in [("nan", [1.0, np.nan, 2.0]), ("inf", [1.0, np.inf, -3.0]), ("neg_inf", [-np.inf, 0.5])]:
        p = Parameter(nt.tensor(np.zeros(len(values), np.float32)))
        p._grad = nt.tensor(np.asarray(values, np.float32))
        norm = nt_optim.get_grad_norm([p])
        specials[name] = float(np.asarray(norm._data)).hex()
    return {"grad_rule": "round_to_bf16(outlier_grads(CONFIG_SMALL, seed=2)) as float32", "cases": cases,
            "specials": specials}


def config2_small(ref) -> dict:
    """Clip at 1.0 + AdamW for 3 steps on bf16-valued outlier gradients (config 2 recipe on the small shapes)."""
    return _config2(ref, W.CONFIG_SMALL, steps=3)


def config2_full(ref) -> dict:
    return _config2(ref, W.CONFIG_124M, steps=2)


def _config2(ref, shape: W.GPTShape, steps: int) -> dict:
    nt, nt_optim, _, Parameter, _ = ref
    params = make_params(nt, Parameter, W.init_params(shape, seed=0))
    opt = nt_optim.AdamW(groups_for(shape, params, W.ADAMW_OPTIONS["weight_decay"]), lr=W.ADAMW_OPTIONS["lr"],
                         betas=W.ADAMW_OPTIONS["betas"], eps=W.ADAMW_OPTIONS["eps"], fused=False)
    norms = []
    t0 = time.perf_counter()
    for step in range(steps):
        grads = [round_to_bf16(g) for g in W.outlier_grads(shape, seed=100 + step)]
        set_grads(nt, params, grads)
        norm = nt_optim.clip_grad_norm_(params, 1.0)
        norms.append(float(np.asarray(norm._data)).hex())
        opt.step()
    seconds = time.perf_counter() - t0
    out = {"config": "2", "shape": shape.name, "steps": steps, "options": W.ADAMW_OPTIONS, "max_norm": 1.0,
           "grad_rule": "round_to_bf16(outlier_grads(shape, seed=100+step))", "norms": norms,
           "numel": shape.numel(), "reference_seconds": seconds}
    out.update(summarize_state(opt, params, copy_dtype="bf16"))
    return out


def xent_cases(ref) -> tuple[dict, dict]:
    nt, _, _, _, F = ref
    cases = {}
    arrays = {}
    rng = np.random.default_rng(11)

    def run(name, logits, targets, sample_cols=None, **kw):
        x = nt.tensor(logits, requires_grad=True)
        t = nt.tensor(targets)
        loss = F.cross_entropy(x, t, **kw)
        if loss.ndim == 0:
            loss.backward()
        else:
            loss.sum().backward()
        grad = np.asarray(x.grad._data)
        loss_np = np.asarray(loss._data)
        entry = {"kwargs": {k: (v if isinstance(v, (int, float, str)) else "tensor") for k, v in kw.items()},
                 "shape": list(logits.shape), "loss_hex": [float(v).hex() for v in np.atleast_1d(loss_np)],
                 "sha256_grad_f32": sha(grad.astype(np.float32)),
                 "sha256_grad_bf16": sha(f32_to_bf16_bits(grad.astype(np.float32)))}
        cases[name] = entry
        if sample_cols is None:
            arrays[name + "__grad"] = grad.astype(np.float32)
        else:
            arrays[name + "__grad_cols"] = grad[:, sample_cols].astype(np.float32)
            arrays[name + "__grad_target"] = grad[np.arange(grad.shape[0]), np.clip(targets, 0, None)].astype(np.float32)
        return entry

    # Config-4 recipe on 64 rows: N(0, 2) logits rounded to bf16, uniform targets.
    logits, targets = W.xent_inputs(rows=64, classes=W.XENT_CLASSES, seed=0)
    logits = round_to_bf16(logits)
    cols = np.arange(0, W.XENT_CLASSES, 97)
    arrays["cols"] = cols
    run("cfg4_64rows_mean", logits, targets, sample_cols=cols)
    t_ign = targets.copy()
    t_ign[::5] = -100
    run("cfg4_64rows_ignore", logits, t_ign, sample_cols=cols)
    weight = rng.uniform(0.5, 1.5, W.XENT_CLASSES).astype(np.float32)
    arrays["cfg4_weight"] = weight
    run("cfg4_64rows_weight_smooth", logits, t_ign, sample_cols=cols, weight=nt.tensor(weight), label_smoothing=0.1)
    run("cfg4_64rows_sum", logits, targets, sample_cols=cols, reduction="sum")
    run("cfg4_64rows_smooth", logits, targets, sample_cols=cols, label_smoothing=0.2)

    # Small explicit cases with edge values.
    small = rng.normal(0, 3, (6, 11)).astype(np.float32)
    small_t = np.array([0, 10, 3, -100, 7, 5], np.int64)
    arrays["small_logits"] = small
    arrays["small_targets"] = small_t
    run("small_mean", small, small_t)
    run("small_none", small, small_t, reduction="none")
    run("small_sum_weight", small, small_t, reduction="sum", weight=nt.tensor(rng.uniform(0.1, 2, 11).astype(np.float32)))
    edge = small.copy()
    edge[1, :] = -np.inf
    edge[2, 4] = np.nan
    edge[4, 1] = np.inf
    edge[5, 2] = -np.inf
    arrays["edge_logits"] = edge
    run("edge_mean", edge, small_t)
    run("all_ignored", small, np.full(6, -100, np.int64))
    return cases, arrays


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("reference", nargs="?", default=os.environ.get("NAMITORCH_REFERENCE",
                                                                       str(REPO.parent / "reference")),
                        help="reference checkout (default: $NAMITORCH_REFERENCE, else ../reference beside this repo)")
    parser.add_argument("--full", action="store_true")
    args = parser.parse_args()
    ref = load_reference(args.reference)
    version = str(getattr(ref[0], "__version__", "unknown"))
    meta = {"reference": "renderityai/NamiTorch", "reference_version": version, "numpy": np.__version__,
            "generator": "tests/golden/make_golden.py"}

    def dump(name, payload):
        (HERE / name).write_text(json.dumps({"meta": meta, **payload}, indent=1, sort_keys=True) + "\n")
        print("wrote", name, flush=True)

    dump("adamw_config0.json", adamw_config0(ref))
    dump("adamw_variants.json", adamw_variants(ref))
    dump("amp_config1.json", amp_config1(ref))
    dump("clip.json", clip_cases(ref))
    dump("config2_small.json", config2_small(ref))
    cases, arrays = xent_cases(ref)
    dump("xent.json", {"cases": cases})
    np.savez_compressed(HERE / "xent_arrays.npz", **arrays)
    print("wrote xent_arrays.npz", flush=True)
    if args.full:
        dump("config2_full.json", config2_full(ref))


if __name__ == "__main__":
    main()
