#!/usr/bin/env python
"""Benchmark of the fused AdamW + AMP optimizer step (and the fused softmax cross-entropy).

Default workload (N = 1): BASELINE configuration 3, the 1.3B-parameter GPT-shaped set
(291 tensors, 1,315,721,216 parameters) with fp32 master weights / moments, a bf16 model
copy and bf16 gradients. One step is the AMP loop of the reference training runner
(namitorch/training/runner.py:247-254) through this package's public API:
    scaler.scale(loss); scaler.unscale_(opt); clip_grad_norm_(params, 1.0);
    scaler.step(opt); scaler.update()
which runs three kernels: gradient statistics (found_inf + norm), the fused multi-tensor
AdamW update (unscale, skip, clip, decoupled decay, moments, bias correction, bf16
cast-out) and the loss-scale update. With N > 1 (torchrun), the same step runs ZeRO-1
sharded: bf16 gradients are reduce-scattered, each rank updates its 1/N shard and the bf16
model copy is all-gathered (NCCL over NVLink); ``value`` is whole-model params/s.

``--workload xent`` times the fused softmax cross-entropy forward + backward on
configuration 4 ([8192, 50257] bf16 logits). ``124m`` and ``small`` run the AMP step on
configurations 2 and 0/1; the step line also reports ``captured`` (the same tail replayed
from one CUDA graph). The kernel seams of the reference's CUDA backend have their own
workloads: ``softmax`` (causal attention softmax, GPT-2 small scores), ``norm`` (layer norm
on 1.3B activations) and ``activation`` (bias + gelu on 1.3B MLP activations).

``--impl reference`` times the reference algorithm on the host CPU (the NumPy oracle port,
all host threads) on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "AdamW+AMP step params/s (achieved HBM GB/s vs B200 peak)"
DEFAULT_PULL = "sm"   # how the ZeRO-1 reduce-scatter reads the peers at N > 1: SM loads or copy engines
FALLBACK_HBM_GBS = 6650.0
BYTES_UPDATE = 28      # adamw_mt: R p4 g2 m4 v4 + W p4 m4 v4 copy2 per parameter
BYTES_STATS = 2        # grad_stats: R g2 per parameter
BYTES_STEP = BYTES_UPDATE + BYTES_STATS


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["1p3b", "124m", "small", "xent", "softmax", "norm", "activation"],
                    default="1p3b")
    ap.add_argument("--softmax-dtype", choices=["f32", "bf16"], default="f32")
    ap.add_argument("--activation-dtype", choices=["f32", "bf16"], default="f32")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--zero-transport", choices=["auto", "p2p", "nccl"], default="auto",
                    help="ZeRO-1 exchange at N>1: fused kernels over peer memory, or NCCL collectives")
    ap.add_argument("--zero-pull", choices=["sm", "copy"], default=DEFAULT_PULL,
                    help="N > 1, p2p transport: the reduce-scatter reads the peers with SM loads or copy engines")
    ap.add_argument("--no-nccl-compare", action="store_true",
                    help="at N>1 with the p2p transport, skip the NCCL-transport comparison run")
    ap.add_argument("--no-extra", action="store_true",
                    help="at N=1, skip the cross-entropy and 124M figures added to the default line")
    return ap.parse_args(argv)


def dist_env():
    return int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("LOCAL_RANK", "0"))


def measured_peak():
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        try:
            data = json.loads(path.read_text())
            return float(data["hbm_gbs"]), "measured"
        except (ValueError, KeyError):
            pass
    return FALLBACK_HBM_GBS, "fallback"


def committed_traffic(kernel: str, workload: str):
    """dram bytes per launch from the committed ncu summary of this kernel/workload, if any."""
    path = REPO / "profiles" / "traffic.json"
    if not path.exists():
        return None
    try:
        return json.loads(path.read_text()).get(f"{kernel}:{workload}")
    except ValueError:
        return None


def pair_traffic(kernel: str, workload: str):
    """Forward + backward dram bytes of one step from the committed ncu summaries, if both exist."""
    fwd = committed_traffic(f"{kernel}_forward", workload)
    bwd = committed_traffic(f"{kernel}_backward", workload)
    return None if fwd is None or bwd is None else {"forward": fwd, "backward": bwd, "step": fwd + bwd}


# ---- clocks sampling --------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str | None):
        self.proc = None
        self.lines: list[str] = []
        cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"]
        if gpu_id:
            cmd += ["-i", gpu_id]
        try:
            self.proc = subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.25)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [[c.strip() for c in line.split(",")] for line in out.splitlines() if line.strip()]
        rows = [r for r in rows if len(r) >= 9]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k].lower() == "active"})
        loaded = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---- CPU baseline (reference algorithm on the host) ------------------------------------------
REFERENCE_INSTALL = REPO / "baseline" / "_ref"
# The CPU sample of the 1.3B workload: layer 0's attention block at d_model 2048 (ln1 weight
# and bias, qkv weight and bias, proj weight and bias), 16,789,504 parameters in two
# parameter groups (decay on the matrices), the same for every CPU figure in a line.
CPU_SAMPLE_SHAPES = [(2048,), (2048,), (2048, 6144), (6144,), (2048, 2048), (2048,)]
CPU_SAMPLE_DECAY = (2, 4)
CPU_SAMPLE_PARAMS = sum(int(np.prod(s)) for s in CPU_SAMPLE_SHAPES)
CPU_SAMPLE_TEXT = (f"{CPU_SAMPLE_PARAMS} parameters (layer 0 attention block of the 1.3B set: ln1 w/b, qkv W/b, "
                   "proj W/b; two groups, wd 0.1 on the matrices), bf16-valued grads x 65536")


def host_info() -> dict:
    """CPU model and the host threads this process may use."""
    model = None
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    usable = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    return {"cpu_model": model, "cpu_count": os.cpu_count(), "usable_threads": usable}


def _cpu_sample_arrays():
    import torch
    rng = np.random.default_rng(0)
    params = [rng.normal(0, 0.02, s).astype(np.float32) for s in CPU_SAMPLE_SHAPES]
    grads = [torch.from_numpy((rng.normal(0, 1e-3, s) * 65536.0).astype(np.float32)).to(torch.bfloat16)
             .to(torch.float32).numpy() for s in CPU_SAMPLE_SHAPES]   # bf16-valued, round to nearest even
    return params, grads


def load_reference_package():
    """The reference installed under baseline/_ref (its own code, unmodified), or None."""
    if not (REFERENCE_INSTALL / "namitorch" / "__init__.py").exists():
        return None
    if str(REFERENCE_INSTALL) not in sys.path:
        sys.path.insert(0, str(REFERENCE_INSTALL))
    import namitorch
    from namitorch import amp, optim
    from namitorch.nn import Parameter
    return namitorch, optim, amp, Parameter


def reference_amp_sample(steps: int, warmup: int = 1) -> dict | None:
    """The reference's own AMP step, through its public API and stock NumPy path
    (namitorch/amp.py:127-234, namitorch/optim/clip_grad.py:96-112, namitorch/optim/adam.py:28-42):
    scaler.scale(loss); scaler.unscale_(opt); clip_grad_norm_(params, 1.0); scaler.step(opt);
    scaler.update(), with AdamW(fused=False) on CPU tensors, over the CPU sample. NumPy runs
    these elementwise passes on one thread. Returns the median per-step throughput of
    `steps` timed steps after `warmup`, or None without the install."""
    ref = load_reference_package()
    if ref is None:
        return None
    nt, optim, amp, Parameter = ref
    params_np, grads_np = _cpu_sample_arrays()
    params = [Parameter(nt.tensor(a)) for a in params_np]
    decay = [params[i] for i in CPU_SAMPLE_DECAY]
    no_decay = [p for i, p in enumerate(params) if i not in CPU_SAMPLE_DECAY]
    opt = optim.AdamW([{"params": decay, "weight_decay": 0.1}, {"params": no_decay, "weight_decay": 0.0}],
                      lr=3e-4, betas=(0.9, 0.999), eps=1e-8, fused=False)
    scaler = amp.GradScaler(init_scale=65536.0, growth_factor=2.0, backoff_factor=0.5, growth_interval=2000)
    loss = nt.tensor(np.float32(1.0))
    times = []
    for k in range(warmup + steps):
        for p, g in zip(params, grads_np):
            p._grad = nt.tensor(g.copy())
        t0 = time.perf_counter()
        scaler.scale(loss)
        scaler.unscale_(opt)
        optim.clip_grad_norm_(params, 1.0)
        scaler.step(opt)
        scaler.update()
        if k >= warmup:
            times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": CPU_SAMPLE_PARAMS / t, "unit": "params/s", "cores": 1, "kind": "reference",
            "sample": CPU_SAMPLE_TEXT + "; the reference's own GradScaler + clip_grad_norm_ 1.0 + AdamW(fused=False) "
                      f"from baseline/_ref (NumPy, one thread), median of {steps} steps after {warmup}",
            "step_seconds": t, "host": host_info()}


def cpu_amp_sample(steps: int, threads: int, warmup: int = 1) -> dict:
    """The oracle port of the same AMP step (unscale, finite, two-pass fp64 norm, clip, AdamW)
    on the same sample, split into per-thread chunks (NumPy ufuncs release the GIL)."""
    from oracle import adamw as oadamw
    params_np, grads_np = _cpu_sample_arrays()
    wd = np.concatenate([np.full(a.size, 0.1 if i in CPU_SAMPLE_DECAY else 0.0) for i, a in enumerate(params_np)])
    p = np.concatenate([a.reshape(-1) for a in params_np])
    g0 = np.concatenate([a.reshape(-1) for a in grads_np])
    n = p.size
    m = np.zeros_like(p)
    v = np.zeros_like(p)
    # chunks never straddle a weight-decay boundary
    edges = np.cumsum([0] + [a.size for a in params_np])
    bounds = []
    chunk = max(1 << 18, n // max(threads, 1) // 4)
    for lo, hi in zip(edges[:-1], edges[1:]):
        bounds += [(i, min(int(hi), i + chunk)) for i in range(int(lo), int(hi), chunk)]
    scale = 65536.0
    pool = ThreadPoolExecutor(max_workers=threads)
    times = []
    step = 0
    for k in range(warmup + steps):
        g = g0.copy()
        t0 = time.perf_counter()

        def unscale(b):
            s, e = b
            np.divide(g[s:e], scale, out=g[s:e])
            return bool(np.all(np.isfinite(g[s:e]))), float(np.max(np.abs(g[s:e]), initial=0))

        parts = list(pool.map(unscale, bounds))
        finite = all(f for f, _ in parts)
        mx = max(x for _, x in parts)

        def sumsq(b):
            s, e = b
            scaled = np.abs(np.asarray(g[s:e], dtype=np.float64)) / mx
            return float(np.sum(np.power(scaled, 2.0), dtype=np.float64))

        total = sum(pool.map(sumsq, bounds))
        norm = mx * math.sqrt(total)
        coef = 1.0 / (norm + 1e-6)
        if finite:
            def clip_and_update(b):
                s, e = b
                if coef < 1:
                    g[s:e] = (np.asarray(g[s:e], np.float64) * coef).astype(np.float32)
                oadamw.adam_update(p[s:e], g[s:e], m[s:e], v[s:e], step, lr=3e-4, beta1=0.9, beta2=0.999,
                                   eps=1e-8, weight_decay=float(wd[s]))

            list(pool.map(clip_and_update, bounds))
            step += 1
        if k >= warmup:
            times.append(time.perf_counter() - t0)
    pool.shutdown()
    t = statistics.median(times)
    return {"value": n / t, "unit": "params/s", "cores": threads, "kind": "port",
            "sample": CPU_SAMPLE_TEXT + "; AMP step = unscale + finite + two-pass fp64 norm + clip 1.0 + AdamW "
                      f"(oracle port, {threads} threads by chunk), median of {steps} steps after {warmup}",
            "step_seconds": t, "host": host_info()}


def cpu_xent_sample(rows: int, threads: int) -> dict:
    from oracle import xent as oxent
    from oracle.casts import round_to_bf16
    from namitorch_b200 import workloads as W
    logits, targets = W.xent_inputs(rows=rows, seed=0)
    logits = round_to_bf16(logits)
    per = max(1, rows // threads)
    blocks = [(i, min(rows, i + per)) for i in range(0, rows, per)]
    t0 = time.perf_counter()
    with ThreadPoolExecutor(max_workers=threads) as pool:
        list(pool.map(lambda b: oxent.cross_entropy(logits[b[0]:b[1]], targets[b[0]:b[1]], reduction="sum"), blocks))
    t = time.perf_counter() - t0
    return {"value": rows / t, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{rows} rows of [8192, 50257] bf16-valued logits, fwd+bwd, row blocks per thread"}


# ---- GPU workloads ---------------------------------------------------------------------------
def shape_for(name):
    from namitorch_b200 import workloads as W
    return {"1p3b": W.CONFIG_1P3B, "124m": W.CONFIG_124M, "small": W.CONFIG_SMALL}[name]


def make_params(shape, device, seed=0):
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    params = []
    for _, s in shape.shapes():
        t = torch.empty(s, dtype=torch.float32, device=device)
        t.normal_(0.0, 0.02, generator=gen)
        params.append(torch.nn.Parameter(t))
    return params


def make_flat_grads(params, device, scale, seed=1):
    """bf16 gradients N(0,1e-3) * scale as views of one flat buffer (64-element aligned)."""
    import torch
    from namitorch_b200.flat import FlatLayout
    layout = FlatLayout.build([p.numel() for p in params])
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    flat = torch.empty(layout.total, dtype=torch.float32, device=device)
    flat.normal_(0.0, 1e-3, generator=gen)
    flat.mul_(scale)
    flat_bf16 = flat.to(torch.bfloat16)
    del flat
    views = [flat_bf16[o:o + p.numel()].view(p.shape) for p, o in zip(params, layout.offsets)]
    return flat_bf16, views


def group_params(shape, params, wd=0.1):
    decay, no_decay = shape.groups()
    return [{"params": [params[i] for i in decay], "weight_decay": wd},
            {"params": [params[i] for i in no_decay], "weight_decay": 0.0}]


def build_step(shape, device, rank, world, transport, seed_params=0, exchange="flags", pull="sm"):
    """(optimizer, scaler, params, flat gradient buffer, loss, step function) of the AMP step
    on `shape`: AdamW (ZeroAdamW over the process group at N > 1) with a bf16 model copy and
    bf16 gradients N(0, 1e-3) x 65536, GradScaler(65536), clip_grad_norm_ 1.0."""
    import torch
    from namitorch_b200 import GradScaler
    from namitorch_b200.optim import AdamW, clip_grad_norm_
    init_scale = 65536.0
    params = make_params(shape, device, seed=seed_params)
    if world > 1:
        from namitorch_b200.zero import ZeroAdamW
        opt = ZeroAdamW(group_params(shape, params), lr=3e-4, betas=(0.9, 0.999), eps=1e-8,
                        model_dtype=torch.bfloat16, transport=transport, exchange=exchange, pull=pull)
        flat_grads = opt.flat_grads
        with torch.no_grad():
            gen = torch.Generator(device=device)
            gen.manual_seed(1 + rank)
            tmp = torch.empty(flat_grads.numel(), dtype=torch.float32, device=device)
            tmp.normal_(0.0, 1e-3, generator=gen)
            flat_grads.copy_(tmp.mul_(init_scale))
            del tmp
    else:
        opt = AdamW(group_params(shape, params), lr=3e-4, betas=(0.9, 0.999), eps=1e-8, model_dtype=torch.bfloat16)
        flat_grads, views = make_flat_grads(params, device, init_scale)
        for prm, g in zip(params, views):
            prm.grad = g
    scaler = GradScaler(init_scale=init_scale, growth_factor=2.0, backoff_factor=0.5, growth_interval=2000)
    loss = torch.ones((), device=device)

    def step():
        scaler.scale(loss)
        scaler.unscale_(opt)
        clip_grad_norm_(params, 1.0)
        scaler.step(opt)
        scaler.update()

    return opt, scaler, params, flat_grads, loss, step


def device_timed(step, steps: int, warmup: int, world: int) -> float:
    """Mean ms per step over `steps` steps after `warmup`, CUDA events on the current stream,
    barriers and synchronisation on both sides, max over ranks."""
    import torch
    import torch.distributed as dist
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        step()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device=torch.cuda.current_device())
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def run_ours(args):
    import torch
    import torch.distributed as dist
    from namitorch_b200 import _native as N
    from namitorch_b200.optim import clip_grad_norm_

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime
        pin_host_threads(local)
        dist.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=300))
    shape = shape_for(args.workload)
    P = shape.numel()
    opt, scaler, params, flat_grads, loss, plain_step = build_step(shape, device, rank, world, args.zero_transport,
                                                                   pull=args.zero_pull)
    stream = torch.cuda.current_stream()
    ev = []
    phases = []   # ZeRO-1: the optimizer's own events (reduce-scatter, stats, update, all-gather tail)

    def step(record=False):
        scaler.scale(loss)
        if record:
            e = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            e[0].record(stream)
            if world > 1:
                opt.timing = True
        scaler.unscale_(opt)
        clip_grad_norm_(params, 1.0)
        if record:
            e[1].record(stream)
        scaler.step(opt)
        if record:
            e[2].record(stream)
            ev.append(e)
            if world > 1:
                phases.append(list(opt.last_events))
                opt.timing = False
        scaler.update()

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    props = torch.cuda.get_device_properties(device)
    sampler = ClockSampler(f"GPU-{props.uuid}" if getattr(props, "uuid", None) else None) if rank == 0 else None
    time.sleep(0.3)
    launches0 = N.launch_count
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    start.record(stream)
    for _ in range(args.steps):
        step(record=True)
    end.record(stream)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches = N.launch_count - launches0
    clocks = sampler.stop() if sampler else None
    ms = start.elapsed_time(end) / args.steps
    stats_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    update_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    breakdown = None
    if world > 1:
        # Events: [rs start, rs end, update start, updates issued on the main stream,
        # all-gathers done, end]; each phase is averaged over the timed steps.
        def span(a, b):
            return statistics.mean(e[a].elapsed_time(e[b]) for e in phases)
        rs_ms, gstats_ms, upd_ms, ag_tail_ms = span(0, 1), span(1, 2), span(2, 3), span(3, 4)
        t = torch.tensor([ms, update_ms, stats_ms, rs_ms, gstats_ms, upd_ms, ag_tail_ms], dtype=torch.float64,
                         device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, update_ms, stats_ms, rs_ms, gstats_ms, upd_ms, ag_tail_ms = t.tolist()
        breakdown = {"reduce_scatter": rs_ms, "global_stats": gstats_ms,
                     "update_with_overlapped_all_gather": upd_ms, "all_gather_tail": ag_tail_ms,
                     "pieces": opt._pieces, "transport": opt.transport}
        update_ms = upd_ms   # the update kernels alone (all-gathers overlap them on the side stream)
    peak, peak_kind = measured_peak()
    shard = P / world
    traffic = committed_traffic("adamw_mt", args.workload)
    result = {
        "metric": METRIC, "value": P / (ms / 1e3), "unit": "params/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": f"{shape.name} AdamW+AMP step (BASELINE config 3; fp32 master/moments, bf16 grads "
                               "and model copy, GradScaler, clip_grad_norm_ 1.0, 2 param groups)",
                   "params": P, "tensors": len(params),
                   "parallelism": (f"zero1-dp{world}-{opt.transport}" + ("-flags" if opt._uses_flags() else "")
                                   + ("-copy-pull" if opt._uses_flags() and opt._pull == "copy" else ""))
                   if world > 1 else "single",
                   "l2": "inputs larger than L2 (30 B/param x 1.3B per step)", "grad_dtype": "bf16",
                   "model_dtype": "bf16"},
        "hbm_gbs_step": BYTES_STEP * shard / (ms / 1e3) / 1e9,
        "kernels_ms": {"grad_stats": stats_ms, "adamw_mt_update": update_ms},
        "roofline": {"bound": "hbm", "achieved": BYTES_UPDATE * shard / (update_ms / 1e3) / 1e9, "peak": peak,
                     "unit": "GB/s", "frac": BYTES_UPDATE * shard / (update_ms / 1e3) / 1e9 / peak,
                     "peak_source": peak_kind, "kernel": "adamw_mt",
                     "algorithmic_bytes_per_launch": BYTES_UPDATE * shard,
                     # DRAM bytes of one launch: the committed ncu capture of the 1.3B update,
                     # at N > 1 scaled to this rank's shard.
                     "traffic": None if traffic is None else traffic / world,
                     "traffic_source": None if traffic is None else
                     "ncu dram read+write of one 1.3B adamw_mt launch (profiles/dram_1p3b.md)"
                     + (f", scaled to the 1/{world} shard" if world > 1 else "")},
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if breakdown:
        result["zero1_breakdown_ms"] = breakdown
        result["nvlink"] = nvlink_section(opt, P, world, ms, breakdown)
        if opt.transport == "p2p":
            # At N > 1 the update kernel also stores the bf16 copy into N - 1 peers: its floor
            # is the longer of its HBM time and its outbound-link time at the push bandwidth
            # measured in this run (the link from N = 4 on).
            result["roofline"]["with_push"] = dict(result["nvlink"]["update_phase"])
    if world == 1:
        # Before the loop measurements below attach a learning-rate schedule to the optimizer.
        result["step_parity"] = single_parity(opt, scaler, params, loss)
        result["loop"] = loop_tail(args, opt, scaler, params, loss)
        result["captured"] = captured_tail(opt, scaler, params, loss)
    if not args.no_e2e:
        result["e2e"] = e2e_ours(args, opt, scaler, params, flat_grads, loss, world)
    if world > 1:
        result["zero_parity"] = zero_parity(opt, scaler, params, loss)
    # The update alone (the HBM-bound part that shards), for the update-scaling figure
    # t_update(1 GPU, P) / max over ranks t_update(N, P/N). At N > 1 this runs last: it
    # advances the optimizer state without exchanges.
    if world > 1:
        dist.barrier()
        t = torch.tensor([opt.benchmark_shard_update(20)], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        only_ms = float(t.item())
    else:
        only_ms = update_ms
    result["update_only"] = {"ms": only_ms, "params_per_s": P / (only_ms / 1e3), "shard_params": shard,
                             "hbm_gbs": BYTES_UPDATE * shard / (only_ms / 1e3) / 1e9,
                             "frac_of_measured_hbm": BYTES_UPDATE * shard / (only_ms / 1e3) / 1e9 / peak}
    if world > 1:
        dist.barrier()
        opt.close()
        del opt, scaler, params, flat_grads, plain_step
        torch.cuda.empty_cache()
        if args.zero_transport == "auto" and not args.no_nccl_compare:
            result["nccl_transport"] = nccl_comparison(shape, device, rank, world)
    else:
        del opt, scaler, params, flat_grads, plain_step
        torch.cuda.empty_cache()
        if args.workload == "1p3b" and not args.no_extra:
            result.update(extra_workloads(args))
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        ref = reference_amp_sample(steps=3)
        port = cpu_amp_sample(3, len(os.sched_getaffinity(0)))
        result["cpu_baseline"] = ref if ref is not None else port
        result["cpu_port"] = port
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def pin_host_threads(local_rank: int) -> None:
    """Restricts this rank's host threads to the CPUs NVML reports as closest to its GPU, so
    that its pinned host buffers are allocated (first touch) in that GPU's NUMA node. Keeps
    the current affinity when NVML is unavailable or reports nothing."""
    try:
        import pynvml
        pynvml.nvmlInit()
        try:
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            index = int(visible.split(",")[local_rank]) if visible else local_rank
            handle = pynvml.nvmlDeviceGetHandleByIndex(index)
            words = pynvml.nvmlDeviceGetCpuAffinity(handle, 16)
        finally:
            pynvml.nvmlShutdown()
        cpus = {w * 64 + b for w, word in enumerate(words) for b in range(64) if (int(word) >> b) & 1}
        cpus &= set(os.sched_getaffinity(0))
        if cpus:
            os.sched_setaffinity(0, cpus)
    except Exception:
        pass


def measure_peer_bandwidth(world: int, rank: int, device, total_bytes: int = 512 << 20, reps: int = 5) -> dict:
    """SM-driven NVLink bandwidth per GPU and direction, measured in this run with the
    access pattern of the ZeRO-1 kernels (plain 32-byte loads and stores, no copy engine,
    no multicast): every rank at once pulls total_bytes / (N - 1) from each peer's buffer
    (inbound, the reduce-scatter), then pushes as much into each peer's buffer (outbound,
    the all-gather). Median of `reps` launches, max over ranks of each launch's time."""
    import torch
    import torch.distributed as dist
    from namitorch_b200 import _native as N
    per = (total_bytes // (world - 1)) // 32 * 32
    buf = torch.zeros(world * per, dtype=torch.uint8, device=device)   # slot 0: own data; slots 1..N-1: inbox
    handles = [None] * world
    dist.all_gather_object(handles, N.ipc_export(buf.data_ptr()))
    peers = {q: N.ipc_open(*handles[q]) for q in range(world) if q != rank}
    base = buf.data_ptr()
    others = [q for q in range(world) if q != rank]

    def inbox(of: int, sender: int) -> int:   # the slot rank `sender` writes in rank `of`'s buffer
        return 1 + (sender if sender < of else sender - 1)

    pull = ([peers[q] for q in others], [base + inbox(rank, q) * per for q in others])
    push = ([base] * len(others), [peers[q] + inbox(q, rank) * per for q in others])
    out = {}
    for name, (src, dst) in (("pull", pull), ("push", push)):
        times = []
        for _ in range(reps + 1):
            torch.cuda.synchronize()
            dist.barrier()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            N.peer_copy(src, dst, per)
            end.record()
            end.synchronize()
            t = torch.tensor([start.elapsed_time(end)], dtype=torch.float64, device=device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            times.append(float(t.item()))
        ms = statistics.median(times[1:])
        out[f"{name}_gbs"] = (world - 1) * per / (ms / 1e3) / 1e9
        out[f"{name}_ms"] = ms
    torch.cuda.synchronize()
    dist.barrier()
    for ptr in peers.values():
        N.ipc_close(ptr)
    dist.barrier()
    del buf
    out["bytes_per_gpu"] = (world - 1) * per
    out["how"] = ("nt_peer_copy, every rank at once: pull = (N-1) peer buffers -> local, push = local -> (N-1) peer "
                  "buffers; 32-byte SM loads/stores; median of %d launches, max over ranks" % reps)
    return out


def nvlink_section(opt, P: int, world: int, ms: float, breakdown: dict) -> dict:
    """The step's NVLink floor against the peer bandwidth measured in this run: the
    reduce-scatter pulls and the all-gather pushes (N-1)/N of the 2-byte buffer per GPU."""
    link_bytes = 2.0 * P * (world - 1) / world          # per phase, per GPU and direction
    bw = measure_peer_bandwidth(world, opt.rank, opt.device)
    floor_ms = (link_bytes / (bw["pull_gbs"] * 1e9) + link_bytes / (bw["push_gbs"] * 1e9)) * 1e3
    # With HBM: the reduce-scatter phase reads the local shard and serves the peers' pulls
    # (2 B x P/N x N) and writes the reduced shard (2 B x P/N); the update phase moves 28 B per
    # shard parameter plus the peers' pushed copies (2 B x P/N x (N - 1)). Each phase takes the
    # longer of its link time and its HBM time at the measured copy bandwidth.
    hbm, _ = measured_peak()
    shard = P / world
    rs_ms = max(link_bytes / (bw["pull_gbs"] * 1e9), 2.0 * shard * (world + 1) / (hbm * 1e9)) * 1e3
    up_ms = max(link_bytes / (bw["push_gbs"] * 1e9), (BYTES_UPDATE + 2.0 * (world - 1)) * shard / (hbm * 1e9)) * 1e3
    rs_gbs = link_bytes / (breakdown["reduce_scatter"] / 1e3) / 1e9
    push_gbs = link_bytes / (breakdown["update_with_overlapped_all_gather"] / 1e3) / 1e9
    return {"bytes_per_gpu_per_phase": link_bytes, "measured": bw,
            "floor_ms": floor_ms, "step_frac_of_floor": floor_ms / ms,
            "floor_with_hbm_ms": rs_ms + up_ms, "step_frac_of_floor_with_hbm": (rs_ms + up_ms) / ms,
            "reduce_scatter_gbs": rs_gbs, "reduce_scatter_frac_of_pull": rs_gbs / bw["pull_gbs"],
            "update_push_gbs": push_gbs, "update_push_frac_of_push": push_gbs / bw["push_gbs"],
            "update_phase": {"floor_ms": up_ms, "frac_of_floor": up_ms / breakdown["update_with_overlapped_all_gather"],
                             "bound": "nvlink" if link_bytes / (bw["push_gbs"] * 1e9) * 1e3 >= up_ms else "hbm"}}


def parity_piece(opt):
    """The largest parameter piece this rank owns: (index in the optimizer's registration
    order, shard offset, length, the parameter). The index is the optimizer's own (its
    parameters group by group), not the model's order, so the parameter and its group's
    weight decay are looked up in `opt.params_list`."""
    if not opt.pieces:
        return 0, 0, 0, None
    i, off, n, _ = max(opt.pieces, key=lambda t: t[2])
    return i, off, n, opt.params_list[i]


def zero_parity(opt, scaler, params, loss) -> dict:
    """One more ZeRO-1 step, checked on every rank after the timed region.

    * copies_equal: the all-gathered bf16 model copy is byte-identical on every rank (SHA-256
      of the whole copy, compared across ranks);
    * reduce_bit_exact: a seeded slice of up to 1M elements of this rank's reduced gradient
      shard equals the float32 sum of every rank's contribution in rank order, divided by N,
      rounded once to bf16 (the contributions are exchanged with an all-to-all);
    * shard_bit_exact: master / exp_avg / exp_avg_sq of that slice after the step equal what
      the reference's own AdamW(fused=False) (baseline/_ref) computes from the pre-step state
      and the reduced gradient after the reference's unscale (g / scale) and clip multiply
      (f32(f64(g) * coef), coef = 1 / (norm + 1e-6)) with the step's global norm. Without
      the reference install, the single-GPU nt_adamw_f32 kernel is the checker instead.
    Returns the result summed / AND-ed over ranks."""
    import hashlib
    import torch
    import torch.distributed as dist
    from namitorch_b200.optim import clip_grad_norm_
    rank, world, device = opt.rank, opt.world, opt.device
    i, off, n, prm = parity_piece(opt)
    m = min(n, 1 << 20)
    rng = np.random.default_rng(1000 + rank)
    start = off + (int(rng.integers(0, n - m + 1)) if n > m else 0)
    gstart = opt._global(start) if m else 0
    meta = [None] * world
    dist.all_gather_object(meta, (gstart, m))
    with torch.no_grad():
        sends = [opt.flat_grads[g:g + k].contiguous() for g, k in meta]
        recvs = [torch.empty(m, dtype=opt.flat_grads.dtype, device=device) for _ in range(world)]
        dist.all_to_all(recvs, sends)
        pre = [t[start:start + m].detach().cpu().numpy().copy() for t in (opt.master, opt.exp_avg, opt.exp_avg_sq)]
        step_count = int(opt.steps[i].item()) if m else 0
        contrib = [r.float().cpu().numpy() for r in recvs]
    scale = scaler.get_scale()
    scaler.scale(loss)
    finite = scaler.unscale_(opt)
    norm_t = clip_grad_norm_(params, 1.0)
    scaler.step(opt)
    scaler.update()
    torch.cuda.synchronize()
    norm = float(norm_t.item())
    stepped = bool(finite)
    with torch.no_grad():
        reduced_bits = opt.grad_shard[start:start + m].view(torch.int16).cpu().numpy()
        post = [t[start:start + m].detach().cpu().numpy().copy() for t in (opt.master, opt.exp_avg, opt.exp_avg_sq)]
        digest = hashlib.sha256()
        chunk = 1 << 27
        for lo in range(0, opt.copy.numel(), chunk):
            digest.update(opt.copy[lo:lo + chunk].view(torch.int16).cpu().numpy().tobytes())
    digests = [None] * world
    dist.all_gather_object(digests, digest.hexdigest())
    # Reduced gradient: f32 rank-order sum, / N (an exact multiply for a power of two), one RNE rounding.
    total = contrib[0].astype(np.float32)
    for c in contrib[1:]:
        total = (total + c).astype(np.float32)
    total = (total / np.float32(world)).astype(np.float32)
    want_bits = torch.from_numpy(total).to(torch.bfloat16).view(torch.int16).numpy()
    reduce_bad = int(np.count_nonzero(want_bits != reduced_bits))
    reduced = torch.from_numpy(reduced_bits.copy()).view(torch.bfloat16).float().numpy()
    group = next((g for g in opt.param_groups if any(q is prm for q in g["params"])), opt.param_groups[0])
    expect, checker = _shard_reference(pre, reduced, scale, norm, step_count, group, stepped, device)
    shard_bad = sum(int(np.count_nonzero(a.view(np.uint32) != b.view(np.uint32))) for a, b in zip(post, expect))
    t = torch.tensor([reduce_bad, shard_bad, m, int(len(set(digests)) == 1), int(stepped)], dtype=torch.float64,
                     device=device)
    sums, mins = t[:3].clone(), t[3:].clone()
    dist.all_reduce(sums, op=dist.ReduceOp.SUM)
    dist.all_reduce(mins, op=dist.ReduceOp.MIN)
    reduce_bad, shard_bad, checked = (int(x) for x in sums.tolist())
    same, stepped_all = (int(x) for x in mins.tolist())
    errors = torch.tensor([opt.exchange_error()], dtype=torch.int32, device=device)
    dist.all_reduce(errors, op=dist.ReduceOp.MAX)
    return {"copies_equal": bool(same), "reduce_bit_exact": reduce_bad == 0, "shard_bit_exact": shard_bad == 0,
            "mismatches": reduce_bad + shard_bad, "elements_checked": checked, "stepped": bool(stepped_all),
            "exchange_errors": int(errors.item()), "exchange": opt._exchange if opt.transport == "p2p" else "nccl",
            "checker": checker, "copy_sha256": digests[0][:16]}


def single_parity(opt, scaler, params, loss, count: int = 1 << 16) -> dict:
    """One more single-GPU step after the timed region, checked on a seeded slice of `count`
    elements of the largest parameter: master / exp_avg / exp_avg_sq after the step must equal
    what the reference's own AdamW(fused=False) (baseline/_ref) computes from the pre-step
    state and gradient, after the reference's unscale and clip multiply with the step's norm;
    and the bf16 model copy must be the round-to-nearest-even of the new master."""
    import torch
    from namitorch_b200.optim import clip_grad_norm_
    engine = opt._engine
    i = max(range(len(engine.params)), key=lambda k: engine.params[k].numel())
    prm = engine.params[i]
    n = min(count, prm.numel())
    start = int(np.random.default_rng(7).integers(0, prm.numel() - n + 1))
    views = [engine.master_view(i), engine.view(engine.exp_avg, i), engine.view(engine.exp_avg_sq, i)]
    with torch.no_grad():
        pre = [v.reshape(-1)[start:start + n].cpu().numpy().copy() for v in views]
        grad = prm.grad.reshape(-1)[start:start + n].float().cpu().numpy()
        step_count = int(engine.steps[i].item())
    scale = scaler.get_scale()
    scaler.scale(loss)
    finite = scaler.unscale_(opt)
    norm_t = clip_grad_norm_(params, 1.0)
    scaler.step(opt)
    scaler.update()
    torch.cuda.synchronize()
    stepped = bool(finite)
    with torch.no_grad():
        post = [v.reshape(-1)[start:start + n].cpu().numpy().copy() for v in views]
        copy_bits = prm.detach().reshape(-1)[start:start + n].view(torch.int16).cpu().numpy()
    group = next(g for g in opt.param_groups if any(q is prm for q in g["params"]))
    expect, checker = _shard_reference(pre, grad, scale, float(norm_t.item()), step_count, group, stepped,
                                       prm.device)
    bad = sum(int(np.count_nonzero(a.view(np.uint32) != b.view(np.uint32))) for a, b in zip(post, expect))
    want_copy = torch.from_numpy(post[0]).to(torch.bfloat16).view(torch.int16).numpy()
    copy_bad = int(np.count_nonzero(want_copy != copy_bits))
    return {"bit_exact": bad == 0 and copy_bad == 0, "mismatches": bad, "copy_mismatches": copy_bad,
            "elements_checked": n, "parameter_index": i, "stepped": stepped, "checker": checker}


def _shard_reference(pre, reduced, scale, norm, step_count, group, stepped, device):
    """(expected master, exp_avg, exp_avg_sq of the slice after the step, checker name)."""
    if not stepped:
        return [a.copy() for a in pre], "skipped step: state unchanged"
    g = (reduced.astype(np.float32) / np.float32(scale)).astype(np.float32)
    coef = 1.0 / (norm + 1e-6)
    if coef < 1:
        g = (g.astype(np.float64) * coef).astype(np.float32)
    lr, (beta1, beta2), eps, wd = group["lr"], group["betas"], group["eps"], group["weight_decay"]
    ref = load_reference_package()
    if ref is not None:
        nt, optim, _, Parameter = ref
        prm = Parameter(nt.tensor(pre[0].copy()))
        ropt = optim.AdamW([{"params": [prm], "weight_decay": wd}], lr=lr, betas=(beta1, beta2), eps=eps, fused=False)
        state = ropt.state_dict()
        if step_count:
            state["state"] = {0: {"step": step_count, "exp_avg": pre[1].copy(), "exp_avg_sq": pre[2].copy()}}
        ropt.load_state_dict(state)
        prm._grad = nt.tensor(g)
        ropt.step()
        st = ropt.state[id(prm)]
        return ([np.asarray(prm._data), np.asarray(st["exp_avg"]._data), np.asarray(st["exp_avg_sq"]._data)],
                "reference AdamW(fused=False) from baseline/_ref")
    import torch
    from namitorch_b200 import _native as N
    from namitorch_b200.optim._common import _scalar
    t = step_count + 1
    coefs = [_scalar(lr), _scalar(beta1), _scalar(beta2), _scalar(1 - beta1), _scalar(1 - beta2), _scalar(eps, "eps"),
             _scalar(wd), _scalar(1 - lr * wd, "decay factor"), _scalar(1 - beta1 ** t), _scalar(1 - beta2 ** t)]
    arrs = [torch.from_numpy(a.copy()).to(device) for a in (pre[0], g, pre[1], pre[2])]
    c = (N.C.c_float * 10)(*[float(x) for x in coefs])
    N.call("nt_adamw_f32", arrs[0].data_ptr(), arrs[1].data_ptr(), arrs[2].data_ptr(), arrs[3].data_ptr(), c, 0,
           int(lr != 0), arrs[0].numel(), N.stream_handle())
    torch.cuda.synchronize()
    return [arrs[k].cpu().numpy() for k in (0, 2, 3)], "nt_adamw_f32 (single-GPU kernel)"


def nccl_comparison(shape, device, rank, world, steps: int = 10, warmup: int = 3) -> dict:
    """The same ZeRO-1 step two more ways, timed the same way, for comparison with the main
    line (peer-memory kernels ordered by in-kernel flags): ``nccl`` is the NCCL transport
    (reduce-scatter, statistics all-reduce, per-piece update + all-gather on a side stream);
    ``p2p_nccl_barriers`` is the peer-memory kernels ordered by NCCL calls between them (two
    4-byte all-reduce barriers and the statistics all-reduce), reading the peers with SM
    loads."""
    import torch
    out = {}
    runs = [("nccl", "nccl", "flags", "sm"), ("p2p_nccl_barriers", "p2p", "nccl", "sm")]
    for name, transport, exchange, pull in runs:
        opt, scaler, params, flat_grads, loss, step = build_step(shape, device, rank, world, transport,
                                                                 exchange=exchange, pull=pull)
        ms = device_timed(step, steps, warmup, world)
        out[name] = {"ms_per_step": ms, "value": shape.numel() / (ms / 1e3), "unit": "params/s", "steps": steps,
                     "warmup": warmup, "pieces": opt._pieces, "transport": opt.transport}
        opt.close()
        del opt, scaler, params, flat_grads, step
        torch.cuda.empty_cache()
    return out


def extra_workloads(args) -> dict:
    """BASELINE configurations 4 (fused cross-entropy, [8192, 50257] bf16) and 2 (the 124M
    AMP step), timed in the same run and added to the default line."""
    import torch
    from namitorch_b200 import workloads as W
    xent = measure_xent(max(20, args.steps), max(3, args.warmup))
    device = torch.device("cuda", torch.cuda.current_device())
    shape = W.CONFIG_124M
    opt, scaler, params, flat_grads, loss, step = build_step(shape, device, 0, 1, "auto")
    ms = device_timed(step, 100, 10, 1)
    peak, _ = measured_peak()
    del opt, scaler, params, flat_grads, step
    torch.cuda.empty_cache()
    return {"xent_ms": xent["ms_per_step"], "xent_frac": xent["roofline"]["frac"],
            "xent_gbs": xent["roofline"]["achieved"],
            "cfg2_ms_per_step": ms, "cfg2_params_per_s": shape.numel() / (ms / 1e3),
            "cfg2_frac": BYTES_STEP * shape.numel() / (ms / 1e3) / 1e9 / peak,
            "extra_what": "xent: BASELINE config 4 fused softmax-CE fwd+bwd, 4 B/logit + 8 B/row; cfg2: BASELINE "
                          "config 2 (124M) AMP step at 30 B/param; CUDA events, measured HBM peak"}


def loop_tail(args, opt, scaler, params, loss, steps: int = 30):
    """The training loop's optimizer tail (namitorch/training/runner.py:247-254) two ways:
    as the reference writes it, reading found_inf, the norm and the step outcome on the host
    each iteration, and with the scheduler gated on the device (no host reads). Device-timed
    with CUDA events around `steps` iterations after 3 warm-up iterations."""
    import torch
    from namitorch_b200.optim import WarmupCosine, clip_grad_norm_

    def synced(sched):
        scaler.scale(loss)
        finite = scaler.unscale_(opt)
        norm = clip_grad_norm_(params, 1.0).item() if finite else None
        updated = scaler.step(opt)
        scaler.update()
        if updated:
            sched.step()
        return norm

    def gated(sched):
        scaler.scale(loss)
        scaler.unscale_(opt)
        clip_grad_norm_(params, 1.0)
        updated = scaler.step(opt)
        scaler.update()
        sched.step(updated)

    out = {}
    for name, body in (("host_reads", synced), ("device_gated", gated)):
        sched = WarmupCosine(opt, warmup_steps=100, total_steps=100000)
        for _ in range(3):
            body(sched)
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            body(sched)
        end.record()
        end.synchronize()
        out[name + "_ms_per_step"] = start.elapsed_time(end) / steps
    out["what"] = ("unscale_ + clip_grad_norm_ + step + update + WarmupCosine step per iteration; host_reads: "
                   "the reference loop's found_inf / norm.item() / `if updated` reads")
    return out


def captured_tail(opt, scaler, params, loss, steps: int = 50):
    """The same AMP step (scale, unscale_, clip_grad_norm_ 1.0, step, update) with the tail
    replayed from one CUDA graph (namitorch_b200.training.CapturedOptimizerStep): one graph
    launch per iteration instead of the tail's host calls. Device-timed with CUDA events over
    `steps` iterations after 3 warm-up replays."""
    import torch
    from namitorch_b200 import _native as N
    from namitorch_b200.training import CapturedOptimizerStep
    step = CapturedOptimizerStep(opt, scaler, params, max_norm=1.0, capacity=steps + 8)
    for _ in range(3):
        scaler.scale(loss)
        step()
    torch.cuda.synchronize()
    launches0 = N.launch_count
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        scaler.scale(loss)
        step()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    return {"ms_per_step": ms, "params_per_s": sum(p.numel() for p in params) / (ms / 1e3),
            "graph_launches_per_step": 1, "host_calls_per_step": "scaler.scale(loss) + one graph replay",
            "what": "scale + unscale_ + clip_grad_norm_ + step + update replayed from one CUDA graph"}


def e2e_ours(args, opt, scaler, params, flat_grads, loss, world):
    """The same step with this step's gradients copied in from pinned host memory and the
    result (norm, found_inf) read back to the host every step, timed on the host clock
    (max over ranks).

    ``serial``: copy, step and read-back one after the other. The reported value is
    ``pipelined``: two device gradient buffers, and the copy of step i + 1's gradients runs
    on a copy stream while step i computes (the prefetch a data loader does); the host still
    reads every step's norm and found_inf before it issues the next step. At N = 1 each
    step's parameters point their ``.grad`` at the buffer its copy landed in; at N > 1 the
    ZeRO-1 optimizer switches between two gradient buffers that every peer has mapped
    (``ZeroAdamW.add_gradient_buffer`` / ``use_gradient_buffer``). Every rank copies its own
    full gradient (data parallelism: each rank's gradients differ). ``h2d_gbs_per_rank`` is
    the copy alone on the copy stream, every rank at once (CUDA events, the slowest rank)."""
    import torch
    import torch.distributed as dist
    from namitorch_b200.optim import clip_grad_norm_
    host = torch.empty(flat_grads.shape, dtype=flat_grads.dtype, pin_memory=True)
    host.copy_(flat_grads)
    out = torch.empty(2, dtype=torch.float64, pin_memory=True)
    nbytes = flat_grads.numel() * flat_grads.element_size()
    P = sum(p.numel() for p in params)
    main = torch.cuda.current_stream()
    side = torch.cuda.Stream(device=flat_grads.device)

    def run_step():
        scaler.scale(loss)
        found = scaler.unscale_(opt)
        norm = clip_grad_norm_(params, 1.0)
        scaler.step(opt)
        scaler.update()
        out[0].copy_(norm, non_blocking=True)
        out[1].copy_(found._tensor, non_blocking=True)

    def slowest(t: float) -> float:
        if world > 1:
            tt = torch.tensor([t], dtype=torch.float64, device=flat_grads.device)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    times = []
    for i in range(args.e2e_steps + 1):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        t0 = time.perf_counter()
        flat_grads.copy_(host, non_blocking=True)
        run_step()
        torch.cuda.current_stream().synchronize()
        if i:
            times.append(time.perf_counter() - t0)
    t_serial = slowest(statistics.median(times))

    # The copy alone: every rank at once, as in the steps.
    copy_ms = []
    for _ in range(3):
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(side):
            e0.record(side)
            flat_grads.copy_(host, non_blocking=True)
            e1.record(side)
        e1.synchronize()
        copy_ms.append(e0.elapsed_time(e1))
    h2d_ms = slowest(statistics.median(copy_ms))

    # Pipelined: buffer b = i % 2 receives step i's gradients on the copy stream; the copy of
    # step i + 1 is queued before step i's compute, behind step i - 1's use of that buffer.
    if world > 1:
        other = opt.add_gradient_buffer() if len(opt.gradient_buffers) < 2 else 1
        bufs = [opt.gradient_buffers[0], opt.gradient_buffers[other]]
        use = [lambda: opt.use_gradient_buffer(0), lambda: opt.use_gradient_buffer(other)]
    else:
        bufs = [flat_grads, torch.empty_like(flat_grads)]
        base = flat_grads.data_ptr()
        grads = [p.grad for p in params]
        views = [[g] for g in grads]
        for g, vs in zip(grads, views):
            off = (g.data_ptr() - base) // flat_grads.element_size()
            vs.append(bufs[1][off:off + g.numel()].view(g.shape))

        def use_views(b):
            for p, vs in zip(params, views):
                p.grad = vs[b]
        use = [lambda: use_views(0), lambda: use_views(1)]
    landed = [torch.cuda.Event() for _ in range(2)]
    released = [torch.cuda.Event() for _ in range(2)]
    steps = args.e2e_steps + 2

    def copy_in(i):
        b = i % 2
        with torch.cuda.stream(side):
            side.wait_event(released[b])
            bufs[b].copy_(host, non_blocking=True)
            landed[b].record(side)

    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    for b in range(2):
        released[b].record(main)
    copy_in(0)
    t1 = time.perf_counter()
    for i in range(steps):
        if i == 1:
            t1 = time.perf_counter()   # the first step (pipeline fill) is not counted
        b = i % 2
        if i + 1 < steps:
            copy_in(i + 1)
        main.wait_event(landed[b])
        use[b]()
        run_step()
        released[b].record(main)
        main.synchronize()              # the host reads step i's norm and found_inf
        _ = float(out[0]), float(out[1])
    t_pipe = slowest((time.perf_counter() - t1) / (steps - 1))
    use[0]()
    torch.cuda.synchronize()
    return {"value": P / t_pipe, "unit": "params/s", "h2d_bytes_per_step": nbytes, "d2h_bytes_per_step": 16,
            "ms_per_step": t_pipe * 1e3, "serial_ms_per_step": t_serial * 1e3, "serial_value": P / t_serial,
            "h2d_ms": h2d_ms, "h2d_gbs_per_rank": nbytes / (h2d_ms / 1e3) / 1e9,
            "host": host_info(),
            "path": "pinned host grads -> H2D on a copy stream (double-buffered, step i+1's copy overlaps step i) "
                    "-> unscale_/clip_grad_norm_/step/update -> D2H norm+found_inf read by the host every step "
                    "(public API); every rank copies its own full gradient"}


def measure_xent(steps: int, warmup: int) -> dict:
    """The fused softmax cross-entropy forward + backward on BASELINE configuration 4."""
    import torch
    from namitorch_b200 import _native as N
    from namitorch_b200 import workloads as W
    from namitorch_b200.nn.functional import softmax_cross_entropy
    device = torch.device("cuda", torch.cuda.current_device())
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    rows, classes = W.XENT_ROWS, W.XENT_CLASSES
    x = torch.empty(rows, classes, dtype=torch.float32, device=device).normal_(0, 2.0, generator=gen).to(torch.bfloat16)
    t = torch.randint(0, classes, (rows,), device=device, generator=gen)
    for _ in range(warmup):
        softmax_cross_entropy(x, t, validate=False)
    torch.cuda.synchronize()
    launches0 = N.launch_count
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(steps):
        loss, dl = softmax_cross_entropy(x, t, validate=False)
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / steps
    peak, kind = measured_peak()
    nbytes = rows * classes * 4 + rows * 8
    result = {"metric": "fused softmax-CE fwd+bwd rows/s", "value": rows / (ms / 1e3), "unit": "rows/s",
              "n_gpus": 1, "steps": steps, "warmup": warmup, "ms_per_step": ms, "higher_is_better": True,
              "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
              "config": {"workload": "LM-head logits [8192, 50257] bf16 N(0,2), int64 targets (BASELINE config 4)",
                         "l2": "inputs larger than L2 (823 MB logits + 823 MB dlogits)"},
              "roofline": {"bound": "hbm", "achieved": nbytes / (ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                           "frac": nbytes / (ms / 1e3) / 1e9 / peak, "peak_source": kind,
                           "traffic": committed_traffic("xent", "xent")},
              "gpu_launches": N.launch_count - launches0}
    del x, t, loss, dl
    torch.cuda.empty_cache()
    return result


def run_xent(args):
    import torch
    torch.cuda.set_device(0)
    result = measure_xent(args.steps, args.warmup)
    if not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_xent_sample(256, os.cpu_count() or 1)
    print(json.dumps(result), flush=True)


def cpu_softmax_sample(rows: int, width: int, threads: int) -> dict:
    """The oracle's causal softmax forward + backward (the reference's arithmetic) on `rows`
    rows of [rows / width, width, width] causal scores, split over host threads (NumPy
    releases the GIL in its ufuncs)."""
    import concurrent.futures as cf
    from oracle import softmax as S
    rng = np.random.default_rng(0)
    x = rng.normal(0, 2, (rows, width)).astype(np.float32)
    g = rng.normal(0, 1, (rows, width)).astype(np.float32)
    per = max(1, -(-rows // threads))

    def part(k):
        lo, hi = k * per, min(rows, (k + 1) * per)
        if lo >= hi:
            return
        xs, gs = x[lo:hi].reshape(1, hi - lo, width), g[lo:hi].reshape(1, hi - lo, width)
        y, _ = S.forward(xs, causal=True, offset=lo % width)
        S.backward(y, gs, causal=True, offset=lo % width)

    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(threads) as pool:
        list(pool.map(part, range(threads)))
    dt = time.perf_counter() - t0
    return {"value": rows / dt, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{rows} rows x {width} causal softmax forward + backward (oracle port of the reference's "
                      "NumPy arithmetic), float32"}


def run_softmax(args):
    """Causal attention softmax forward + backward on GPT-2-small attention scores
    (batch 8 x 12 heads x 1024 queries, 1024 keys): the row-softmax seam's hot shape."""
    import torch
    from namitorch_b200 import _native as N
    from namitorch_b200.backends import get_backend
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    dtype = {"f32": torch.float32, "bf16": torch.bfloat16}[args.softmax_dtype]
    heads, t = 8 * 12, 1024
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    x = torch.randn(heads, t, t, device=device, generator=gen).mul_(2.0).to(dtype)
    g = torch.randn(heads, t, t, device=device, generator=gen).to(dtype)
    k = get_backend(x).softmax
    for _ in range(args.warmup):
        y = k.run("causal_softmax", (x, None))
        k.run("causal_softmax_backward", (y, g, None))
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    launches0 = N.launch_count
    ev[0].record()
    for _ in range(args.steps):
        y = k.run("causal_softmax", (x, None))
    ev[1].record()
    for _ in range(args.steps):
        k.run("causal_softmax_backward", (y, g, None))
    ev[2].record()
    torch.cuda.synchronize()
    fwd, bwd = ev[0].elapsed_time(ev[1]) / args.steps, ev[1].elapsed_time(ev[2]) / args.steps
    elems, es = x.numel(), x.element_size()
    peak, kind = measured_peak()
    rows = heads * t
    # The causal forward reads only the allowed scores (t (t + 1) / 2 of a head's t^2; the
    # masked part is never used) and writes every output; the backward reads y and g whole.
    allowed = heads * t * (t + 1) // 2
    fwd_bytes, bwd_bytes = es * (allowed + elems), 3 * es * elems
    achieved = (fwd_bytes + bwd_bytes) / ((fwd + bwd) / 1e3) / 1e9
    result = {"metric": "causal attention softmax fwd+bwd rows/s", "value": rows / ((fwd + bwd) / 1e3),
              "unit": "rows/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": fwd + bwd,
              "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": args.softmax_dtype,
              "data": "synthetic",
              "config": {"workload": f"attention scores [{heads} x {t}, {t}] N(0,2), causal (GPT-2 small, batch 8)",
                         "l2": f"inputs larger than L2 ({elems * es / 1e6:.0f} MB per tensor)"},
              "kernels_ms": {"forward": fwd, "backward": bwd},
              "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                           "peak_source": kind,
                           "algorithmic_bytes": {"forward": fwd_bytes, "backward": bwd_bytes},
                           "forward_gbs": fwd_bytes / (fwd / 1e3) / 1e9,
                           "backward_gbs": bwd_bytes / (bwd / 1e3) / 1e9,
                           "traffic": pair_traffic("row_softmax", f"softmax_{args.softmax_dtype}")},
              "gpu_launches": N.launch_count - launches0}
    if not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_softmax_sample(4096, t, os.cpu_count() or 1)
    print(json.dumps(result), flush=True)


def cpu_norm_sample(rows: int, width: int, threads: int) -> dict:
    """The oracle's layer norm forward + backward (input, weight and bias gradients; the
    reference's arithmetic) on `rows` rows of `width`, split over host threads."""
    import concurrent.futures as cf
    from oracle import normalization as O
    rng = np.random.default_rng(0)
    x = (rng.normal(0, 2, (rows, width)) + 1).astype(np.float32)
    g = rng.normal(0, 1, (rows, width)).astype(np.float32)
    w = (rng.normal(0, 0.1, width) + 1).astype(np.float32)
    b = rng.normal(0, 0.1, width).astype(np.float32)
    per = max(1, -(-rows // threads))

    def part(k):
        lo, hi = k * per, min(rows, (k + 1) * per)
        if lo >= hi:
            return
        _, stats = O.forward(x[lo:hi], w, b, 1e-5, True)
        O.backward(x[lo:hi], w, g[lo:hi], stats, True)

    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(threads) as pool:
        list(pool.map(part, range(threads)))
    dt = time.perf_counter() - t0
    return {"value": rows / dt, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{rows} rows x {width} layer norm forward + backward with weight and bias (oracle port of "
                      "the reference's NumPy arithmetic), float32"}


def run_norm(args):
    """Layer norm forward + backward (input, weight and bias gradients) on the 1.3B model's
    activations: 16 sequences x 2048 tokens x d_model 2048, float32."""
    import torch
    from namitorch_b200 import _native as N
    from namitorch_b200.backends import get_backend
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    rows, width = 16 * 2048, 2048
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    x = torch.randn(rows, width, device=device, generator=gen).mul_(2.0).add_(1.0)
    g = torch.randn(rows, width, device=device, generator=gen)
    w = torch.randn(width, device=device, generator=gen).mul_(0.1).add_(1.0)
    b = torch.randn(width, device=device, generator=gen).mul_(0.1)
    k = get_backend(x).normalization
    for _ in range(args.warmup):
        y, st = k.run("layer_norm", (x, w, b), eps=1e-5)
        k.run("layer_norm_backward", (x, w, g, st))
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    launches0 = N.launch_count
    ev[0].record()
    for _ in range(args.steps):
        y, st = k.run("layer_norm", (x, w, b), eps=1e-5)
    ev[1].record()
    for _ in range(args.steps):
        k.run("layer_norm_backward", (x, w, g, st))
    ev[2].record()
    torch.cuda.synchronize()
    fwd, bwd = ev[0].elapsed_time(ev[1]) / args.steps, ev[1].elapsed_time(ev[2]) / args.steps
    elems = x.numel()
    peak, kind = measured_peak()
    achieved = (8 + 12) * elems / ((fwd + bwd) / 1e3) / 1e9
    result = {"metric": "layer norm fwd+bwd rows/s", "value": rows / ((fwd + bwd) / 1e3), "unit": "rows/s",
              "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": fwd + bwd,
              "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
              "data": "synthetic",
              "config": {"workload": f"activations [{rows}, {width}] (1.3B model, 16 x 2048 tokens), weight and bias",
                         "l2": f"inputs larger than L2 ({elems * 4 / 1e6:.0f} MB per tensor)"},
              "kernels_ms": {"forward": fwd, "backward": bwd},
              "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                           "peak_source": kind,
                           "algorithmic_bytes": {"forward": 8 * elems, "backward": 12 * elems},
                           "forward_gbs": 8 * elems / (fwd / 1e3) / 1e9, "backward_gbs": 12 * elems / (bwd / 1e3) / 1e9,
                           "traffic": pair_traffic("norm", "norm")},
              "gpu_launches": N.launch_count - launches0}
    if not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_norm_sample(8192, width, os.cpu_count() or 1)
    print(json.dumps(result), flush=True)


def cpu_activation_sample(rows: int, width: int, threads: int) -> dict:
    """The oracle's bias + gelu(tanh) forward and backward (the reference's arithmetic) on
    `rows` rows of `width`, split over host threads."""
    import concurrent.futures as cf
    from oracle import activations as A
    rng = np.random.default_rng(0)
    x = rng.normal(0, 1, (rows, width)).astype(np.float32)
    g = rng.normal(0, 1, (rows, width)).astype(np.float32)
    b = rng.normal(0, 0.1, width).astype(np.float32)
    per = max(1, -(-rows // threads))

    def part(k):
        lo, hi = k * per, min(rows, (k + 1) * per)
        if lo < hi:
            A.apply("bias_gelu_tanh", (x[lo:hi], b))
            A.apply("bias_gelu_tanh_backward", (x[lo:hi], b, g[lo:hi]))

    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(threads) as pool:
        list(pool.map(part, range(threads)))
    dt = time.perf_counter() - t0
    return {"value": rows / dt, "unit": "rows/s", "cores": threads, "kind": "port",
            "sample": f"{rows} rows x {width} bias + gelu(tanh) forward + backward (oracle port of the reference's "
                      "NumPy arithmetic), float32"}


def run_activation(args):
    """bias + gelu(tanh) forward and backward (the fused-elementwise seam) on the 1.3B model's
    MLP activations: 16 sequences x 2048 tokens x 8192 hidden, float32 or bfloat16
    (--activation-dtype)."""
    import torch
    from namitorch_b200 import _native as N
    from namitorch_b200.backends import get_backend
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    rows, width = 16 * 2048, 4 * 2048
    gen = torch.Generator(device=device)
    gen.manual_seed(0)
    dtype = {"f32": torch.float32, "bf16": torch.bfloat16}[args.activation_dtype]
    x = torch.randn(rows, width, device=device, generator=gen).to(dtype)
    g = torch.randn(rows, width, device=device, generator=gen).to(dtype)
    b = torch.randn(width, device=device, generator=gen).mul_(0.1).to(dtype)
    k = get_backend(x).fused
    for _ in range(args.warmup):
        k.run("bias_gelu_tanh", (x, b))
        k.run("bias_gelu_tanh_backward", (x, b, g))
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    launches0 = N.launch_count
    ev[0].record()
    for _ in range(args.steps):
        k.run("bias_gelu_tanh", (x, b))
    ev[1].record()
    for _ in range(args.steps):
        k.run("bias_gelu_tanh_backward", (x, b, g))
    ev[2].record()
    torch.cuda.synchronize()
    fwd, bwd = ev[0].elapsed_time(ev[1]) / args.steps, ev[1].elapsed_time(ev[2]) / args.steps
    elems, es = x.numel(), x.element_size()
    peak, kind = measured_peak()
    # forward R x + W y, backward R x, g + W dx per element (the bias row stays in cache)
    fwd_bytes, bwd_bytes = 2 * es * elems, 3 * es * elems
    achieved = (fwd_bytes + bwd_bytes) / ((fwd + bwd) / 1e3) / 1e9
    result = {"metric": "bias+gelu(tanh) fwd+bwd rows/s", "value": rows / ((fwd + bwd) / 1e3), "unit": "rows/s",
              "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": fwd + bwd,
              "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": args.activation_dtype,
              "data": "synthetic",
              "config": {"workload": f"MLP activations [{rows}, {width}] (1.3B model, 16 x 2048 tokens), bias [{width}]",
                         "l2": f"inputs larger than L2 ({elems * es / 1e6:.0f} MB per tensor)"},
              "kernels_ms": {"forward": fwd, "backward": bwd},
              "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                           "peak_source": kind,
                           "algorithmic_bytes": {"forward": fwd_bytes, "backward": bwd_bytes},
                           "forward_gbs": fwd_bytes / (fwd / 1e3) / 1e9, "backward_gbs": bwd_bytes / (bwd / 1e3) / 1e9,
                           "traffic": pair_traffic("fused_bias_gelu", "activation") if es == 4 else None},
              "gpu_launches": N.launch_count - launches0}
    if not args.no_cpu_baseline:
        result["cpu_baseline"] = cpu_activation_sample(2048, width, os.cpu_count() or 1)
    print(json.dumps(result), flush=True)


def run_reference(args):
    rank, world, _ = dist_env()
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0))
    if args.workload == "xent":
        times = []
        for i in range(args.warmup + args.steps):
            base = cpu_xent_sample(128, threads)
            if i >= args.warmup:
                times.append(base["value"])
        value = statistics.median(times)
        base["value"] = value
        line = {"impl": "reference", "metric": "fused softmax-CE fwd+bwd rows/s", "value": value, "unit": "rows/s",
                "higher_is_better": True}
    elif args.workload == "softmax":
        times = []
        for i in range(args.warmup + args.steps):
            base = cpu_softmax_sample(2048, 1024, threads)
            if i >= args.warmup:
                times.append(base["value"])
        value = statistics.median(times)
        base["value"] = value
        line = {"impl": "reference", "metric": "causal attention softmax fwd+bwd rows/s", "value": value,
                "unit": "rows/s", "higher_is_better": True}
    elif args.workload == "activation":
        times = []
        for i in range(args.warmup + args.steps):
            base = cpu_activation_sample(1024, 8192, threads)
            if i >= args.warmup:
                times.append(base["value"])
        value = statistics.median(times)
        base["value"] = value
        line = {"impl": "reference", "metric": "bias+gelu(tanh) fwd+bwd rows/s", "value": value, "unit": "rows/s",
                "higher_is_better": True}
    elif args.workload == "norm":
        times = []
        for i in range(args.warmup + args.steps):
            base = cpu_norm_sample(4096, 2048, threads)
            if i >= args.warmup:
                times.append(base["value"])
        value = statistics.median(times)
        base["value"] = value
        line = {"impl": "reference", "metric": "layer norm fwd+bwd rows/s", "value": value, "unit": "rows/s",
                "higher_is_better": True}
    else:
        # The reference's own AMP step (baseline/_ref, its public API and NumPy path) on the
        # CPU sample; the threaded oracle port of the same step beside it.
        base = reference_amp_sample(steps=args.steps, warmup=args.warmup)
        port = cpu_amp_sample(args.steps, threads, warmup=args.warmup)
        if base is None:
            base = dict(port, note="baseline/_ref is not installed: the oracle port stands in for the reference")
        value = base["value"]
        line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "params/s", "higher_is_better": True,
                "port_threaded": {k: port[k] for k in ("value", "unit", "cores", "kind", "sample")},
                "host": base.get("host")}
    line.update({"n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                 "config": {"workload": args.workload, "sample": base["sample"]},
                 "cpu_baseline": {k: base[k] for k in ("value", "unit", "cores", "kind", "sample")},
                 "e2e": {"value": value, "unit": line["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                 "dtype": "f32", "data": "synthetic", "scaling": "strong", "vs_baseline": None})
    print(json.dumps(line), flush=True)


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
        return
    if args.workload == "xent":
        run_xent(args)
        return
    if args.workload == "softmax":
        run_softmax(args)
        return
    if args.workload == "norm":
        run_norm(args)
        return
    if args.workload == "activation":
        run_activation(args)
        return
    run_ours(args)


if __name__ == "__main__":
    main()
