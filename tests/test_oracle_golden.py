"""Pins the CPU oracle against fixtures produced by running the reference itself.

Every fixture in tests/golden was written by tests/golden/make_golden.py from the
reference's own public API; these tests re-derive each result with ``oracle`` and require
bit-identical float32 / float16 / bfloat16 bytes (SHA-256) for the optimizer, scaler and
clipping paths and tight tolerances for cross-entropy (whose reductions are summed in a
different order).
"""
import hashlib
import math

import numpy as np
import pytest

from conftest import GOLDEN, load_golden
from namitorch_b200 import workloads as W
from oracle import adamw as oadamw
from oracle import amp as oamp
from oracle import clip as oclip
from oracle import xent as oxent
from oracle.casts import f32_to_bf16_bits, round_to_bf16


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def oracle_optimizer(shape, params, options=W.ADAMW_OPTIONS):
    decay, no_decay = shape.groups()
    base = {"lr": options["lr"], "betas": options["betas"], "eps": options["eps"], "maximize": False}
    groups = [(decay, {**base, "weight_decay": options["weight_decay"]}), (no_decay, {**base, "weight_decay": 0.0})]
    return oadamw.OracleAdamW(params, groups)


def check_state(opt, params, gold, copy=None):
    ps = params
    ms = [opt.state[i]["exp_avg"] for i in range(len(params)) if i in opt.state]
    vs = [opt.state[i]["exp_avg_sq"] for i in range(len(params)) if i in opt.state]
    assert [opt.state.get(i, {}).get("step", 0) for i in range(len(params))] == gold["param_steps"]
    assert [sha(p) for p in ps] == gold["per_tensor_sha256_param"]
    assert sha(*ps) == gold["sha256_param"]
    assert sha(*ms) == gold["sha256_exp_avg"]
    assert sha(*vs) == gold["sha256_exp_avg_sq"]
    if copy == "f16":
        assert sha(*[p.astype(np.float16) for p in ps]) == gold["sha256_copy_f16"]
    if copy == "bf16":
        assert sha(*[f32_to_bf16_bits(p) for p in ps]) == gold["sha256_copy_bf16"]


def test_adamw_config0_bit_exact():
    gold = load_golden("adamw_config0.json")
    shape = W.CONFIG_SMALL
    params = W.init_params(shape, seed=0)
    opt = oracle_optimizer(shape, params)
    grads = W.normal_grads(shape, seed=0)
    for _ in range(gold["steps"]):
        opt.step([g.copy() for g in grads])
    check_state(opt, params, gold)


@pytest.mark.parametrize("case", ["adamw_default", "adamw_maximize", "adamw_lr0", "adamw_wd0", "adam_coupled",
                                  "adam_betas"])
def test_adamw_variants_bit_exact(case):
    gold = load_golden("adamw_variants.json")
    c = gold["cases"][case]
    o = c["options"]
    p = np.asarray(gold["base_param"], np.uint32).view(np.float32).reshape(gold["shape"]).copy()
    g0 = np.asarray(gold["base_grad"], np.uint32).view(np.float32).reshape(gold["shape"])
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    step = 0
    for k in range(gold["steps"]):
        with np.errstate(all="ignore"):
            step = oadamw.adam_update(p, (g0 * (k + 1)).astype(np.float32), m, v, step, lr=o["lr"],
                                      beta1=o["betas"][0], beta2=o["betas"][1], eps=o["eps"],
                                      weight_decay=o["weight_decay"], maximize=o["maximize"],
                                      decoupled=o["cls"] == "AdamW")
    assert step == c["step"]
    assert p.view(np.uint32).reshape(-1).tolist() == c["param"]
    assert m.view(np.uint32).reshape(-1).tolist() == c["exp_avg"]
    assert v.view(np.uint32).reshape(-1).tolist() == c["exp_avg_sq"]


def test_amp_config1_trajectory_bit_exact():
    gold = load_golden("amp_config1.json")
    shape = W.CONFIG_SMALL
    params = W.init_params(shape, seed=0)
    opt = oracle_optimizer(shape, params)
    s = gold["scaler"]
    scaler = oamp.OracleGradScaler(s["init_scale"], s["growth_factor"], s["backoff_factor"], s["growth_interval"])
    inf_idx = W.inf_positions(shape.shapes()[0][1][0] * shape.shapes()[0][1][1], 0.001, seed=0)
    assert inf_idx.size == gold["inf_count"]
    for step, expected in enumerate(gold["trace"]):
        base = W.normal_grads(shape, seed=1000 + step)
        g16 = [(g * np.float32(scaler.scale)).astype(np.float16) for g in base]
        if step == 3:
            g16[0].reshape(-1)[inf_idx] = np.float16(np.inf)
        grads = [g.astype(np.float32) for g in g16]
        r = oamp.amp_step(opt, scaler, grads)
        assert float(r["scale_used"]).hex() == expected["scale_used"]
        assert r["stepped"] == expected["stepped"] == expected["finite"]
        assert float(r["scale_after"]).hex() == expected["scale_after"]
        assert r["growth_tracker"] == expected["growth_tracker"]
    check_state(opt, params, gold, copy="f16")


@pytest.mark.parametrize("name", ["bf16_outliers_p2", "bf16_outliers_pinf", "bf16_outliers_p1",
                                  "bf16_outliers_p3.5", "small_noclip_p2", "zeros_p2"])
def test_clip_cases_bit_exact(name):
    gold = load_golden("clip.json")
    c = gold["cases"][name]
    base = [round_to_bf16(g) for g in W.outlier_grads(W.CONFIG_SMALL, seed=2)]
    if name.startswith("small"):
        grads = [g * np.float32(1e-3) for g in base]
    elif name.startswith("zeros"):
        grads = [np.zeros_like(g) for g in base[:3]]
    else:
        grads = [g.copy() for g in base]
    norm = oclip.clip_grad_norm_(grads, c["max_norm"], c["norm_type"])
    assert float(norm).hex() == c["norm"]
    assert sha(*grads) == c["sha256_clipped"]


def test_clip_specials():
    gold = load_golden("clip.json")["specials"]
    assert math.isnan(float.fromhex(gold["nan"])) and math.isnan(float(oclip.total_norm([np.array([1, np.nan, 2], np.float32)])))
    assert float(oclip.total_norm([np.array([1, np.inf, -3], np.float32)])).hex() == gold["inf"]
    assert float(oclip.total_norm([np.array([-np.inf, 0.5], np.float32)])).hex() == gold["neg_inf"]


def test_config2_small_bit_exact():
    gold = load_golden("config2_small.json")
    shape = W.CONFIG_SMALL
    params = W.init_params(shape, seed=0)
    opt = oracle_optimizer(shape, params)
    for step in range(gold["steps"]):
        grads = [round_to_bf16(g) for g in W.outlier_grads(shape, seed=100 + step)]
        norm = oclip.clip_grad_norm_(grads, gold["max_norm"])
        assert float(norm).hex() == gold["norms"][step]
        opt.step(grads)
    check_state(opt, params, gold, copy="bf16")


@pytest.mark.slow
@pytest.mark.skipif(not (GOLDEN / "config2_full.json").exists(), reason="full config-2 fixture not generated")
def test_config2_full_bit_exact():
    gold = load_golden("config2_full.json")
    shape = W.CONFIG_124M
    params = W.init_params(shape, seed=0)
    opt = oracle_optimizer(shape, params)
    for step in range(gold["steps"]):
        grads = [round_to_bf16(g) for g in W.outlier_grads(shape, seed=100 + step)]
        norm = oclip.clip_grad_norm_(grads, gold["max_norm"])
        assert float(norm).hex() == gold["norms"][step]
        opt.step(grads)
    check_state(opt, params, gold, copy="bf16")


def _xent_case(name):
    gold = load_golden("xent.json")["cases"][name]
    arrays = np.load(GOLDEN / "xent_arrays.npz")
    return gold, arrays


@pytest.mark.parametrize("name,kwargs,targets_fn", [
    ("cfg4_64rows_mean", {}, lambda t: t),
    ("cfg4_64rows_ignore", {}, lambda t: np.where(np.arange(t.size) % 5 == 0, -100, t)),
    ("cfg4_64rows_weight_smooth", {"weight": True, "label_smoothing": 0.1},
     lambda t: np.where(np.arange(t.size) % 5 == 0, -100, t)),
    ("cfg4_64rows_sum", {"reduction": "sum"}, lambda t: t),
    ("cfg4_64rows_smooth", {"label_smoothing": 0.2}, lambda t: t),
])
def test_xent_cfg4_rows(name, kwargs, targets_fn):
    gold, arrays = _xent_case(name)
    logits, targets = W.xent_inputs(rows=64, classes=W.XENT_CLASSES, seed=0)
    logits = round_to_bf16(logits)
    targets = targets_fn(targets)
    kw = dict(kwargs)
    if kw.pop("weight", False):
        kw["weight"] = arrays["cfg4_weight"]
    loss, grad = oxent.cross_entropy(logits, targets, **kw)
    ref_loss = float.fromhex(gold["loss_hex"][0])
    assert abs(float(loss) - ref_loss) <= 2e-6 * abs(ref_loss)
    cols = arrays["cols"]
    np.testing.assert_allclose(grad[:, cols], arrays[name + "__grad_cols"], rtol=2e-5, atol=1e-12)
    tcol = grad[np.arange(64), np.clip(targets, 0, None)]
    np.testing.assert_allclose(tcol, arrays[name + "__grad_target"], rtol=2e-5, atol=1e-12)


@pytest.mark.parametrize("name", ["small_mean", "small_none", "edge_mean", "all_ignored"])
def test_xent_small(name):
    gold, arrays = _xent_case(name)
    logits = arrays["edge_logits"] if name.startswith("edge") else arrays["small_logits"]
    targets = np.full(6, -100, np.int64) if name == "all_ignored" else arrays["small_targets"]
    kw = {"reduction": "none"} if name == "small_none" else {}
    with np.errstate(all="ignore"):
        loss, grad = oxent.cross_entropy(logits, targets, **kw)
    ref = np.array([float.fromhex(h) for h in gold["loss_hex"]], np.float32)
    np.testing.assert_allclose(np.atleast_1d(loss), ref, rtol=2e-6, atol=0, equal_nan=True)
    np.testing.assert_allclose(grad, arrays[name + "__grad"], rtol=2e-5, atol=1e-9, equal_nan=True)


def test_bf16_rounding_matches_ml_dtypes():
    ml_dtypes = pytest.importorskip("ml_dtypes")
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.normal(0, 1, 10000).astype(np.float32),
                        np.array([0.0, -0.0, 1e-40, -1e-41, 3.4e38, -3.4e38, np.inf, -np.inf,
                                  1.00390625, 1.01171875, 1.0078125], np.float32)])
    ours = f32_to_bf16_bits(x)
    theirs = x.astype(ml_dtypes.bfloat16).view(np.uint16)
    assert np.array_equal(ours, theirs)
