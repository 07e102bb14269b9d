"""ZeRO-1 on 2+ GPUs: one process per GPU, GradScaler + clip_grad_norm_ + AdamW, over both
transports (NCCL collectives; the fused kernels over peer memory, ordered across GPUs by
flags inside the kernels or by NCCL calls between them).

The oracle receives the gradients as they come out of the reduce-scatter (gathered from
every rank), so the comparison isolates the sharded update from the bf16 reduction
rounding; the reduction itself is checked against a float32 sum within bf16 rounding.
Skipped when fewer than two GPUs are visible.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# Ranks (one GPU each); NT_ZERO_TEST_WORLD raises it on a box with more GPUs.
WORLD = int(os.environ.get("NT_ZERO_TEST_WORLD", "2"))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _round_to(dtype: str):
    """float32 -> the model dtype (round to nearest even) -> float32."""
    from oracle.casts import round_to_bf16
    if dtype == "f16":
        return lambda x: np.asarray(x, np.float32).astype(np.float16).astype(np.float32)
    return round_to_bf16


def _worker(rank, world, port, out_path, transport, lazy, exchange, norm_type=2.0, dtype="bf16", pull="sm"):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from namitorch_b200 import GradScaler, workloads as W
        from namitorch_b200.optim import clip_grad_norm_, defer_gradient_transforms
        from namitorch_b200.zero import ZeroAdamW
        defer_gradient_transforms(lazy)
        round_grad = _round_to(dtype)
        model_dtype = torch.float16 if dtype == "f16" else torch.bfloat16
        shape = W.CONFIG_SMALL
        params = [torch.nn.Parameter(torch.from_numpy(a).cuda()) for a in W.init_params(shape, seed=0)]
        decay, no_decay = shape.groups()
        groups = [{"params": [params[i] for i in decay], "weight_decay": 0.1},
                  {"params": [params[i] for i in no_decay], "weight_decay": 0.0}]
        opt = ZeroAdamW(groups, lr=3e-4, model_dtype=model_dtype, transport=transport, exchange=exchange, pull=pull)
        assert opt.transport == transport
        scaler = GradScaler(1024.0, growth_interval=2)
        reduced, local, norms, stepped = [], [], [], []
        for step in range(4):
            opt.zero_grad()
            grads = [round_grad(g * np.float32(scaler.get_scale()))
                     for g in W.outlier_grads(shape, seed=10 * step + rank)]
            if step == 2 and rank == 1:
                grads[5].reshape(-1)[3] = np.inf
            for p, g in zip(params, grads):
                p.grad.copy_(torch.from_numpy(g).to(model_dtype))
            local.append(opt.flat_grads.float().cpu().numpy())
            if not lazy:
                # The eager path rewrites the reduced shard in place: read it before.
                opt._reduce()
                reduced.append(opt._gather_shards(opt.grad_shard).float().cpu().numpy())
            scaler.scale(torch.ones((), device="cuda"))
            scaler.unscale_(opt)
            norms.append(float(clip_grad_norm_(params, 1.0, norm_type=norm_type).item()))
            stepped.append(bool(scaler.step(opt)))
            scaler.update()
            if lazy:
                # Deferred transforms leave the reduced shard as the reduce-scatter wrote it.
                reduced.append(opt._gather_shards(opt.grad_shard).float().cpu().numpy())
        opt.check_exchange()   # no in-kernel wait on another rank ran out
        sd = opt.state_dict()
        copies = [p.detach().float().cpu().numpy() for p in params]
        all_local = [None] * world
        dist.all_gather_object(all_local, local)
        if rank == 0:
            np.savez(out_path, norms=np.array(norms), stepped=np.array(stepped),
                     offsets=np.array(opt.layout.offsets), reduced=np.stack(reduced),
                     local=np.stack([np.stack(l) for l in all_local]),
                     **{f"master{k}": st["master_param"].cpu().numpy() for k, st in sd["state"].items()},
                     **{f"m{k}": st["exp_avg"].cpu().numpy() for k, st in sd["state"].items()},
                     steps=np.array([st["step"] for _, st in sorted(sd["state"].items())]),
                     **{f"copy{k}": c for k, c in enumerate(copies)}, scale=np.array(scaler.get_scale()))
        dist.barrier()
        opt.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("transport,lazy,exchange,norm_type,dtype,pull", [
    ("nccl", True, "flags", 2.0, "bf16", "sm"), ("p2p", True, "flags", 2.0, "bf16", "sm"),
    ("p2p", False, "flags", 2.0, "bf16", "sm"), ("p2p", True, "nccl", 2.0, "bf16", "sm"),
    ("p2p", True, "flags", float("inf"), "bf16", "sm"), ("p2p", True, "flags", 3.0, "bf16", "sm"),
    ("p2p", False, "flags", 2.0, "f16", "sm"), ("p2p", True, "flags", 2.0, "bf16", "copy"),
    ("p2p", False, "flags", float("inf"), "f16", "copy")])
def test_zero1_matches_oracle(tmp_path, transport, lazy, exchange, norm_type, dtype, pull):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp
    from namitorch_b200 import workloads as W
    from oracle import adamw as oadamw
    from oracle import amp as oamp
    from oracle import clip as oclip
    out_path = tmp_path / "zero.npz"
    mp.spawn(_worker, args=(WORLD, _free_port(), str(out_path), transport, lazy, exchange, norm_type, dtype, pull),
             nprocs=WORLD, join=True)
    round_model = _round_to(dtype)
    out = np.load(out_path)
    shape = W.CONFIG_SMALL
    offsets = out["offsets"]
    numels = [int(np.prod(s)) for _, s in shape.shapes()]
    # The reduce-scatter (average) agrees with a float32 mean within bf16 rounding. NCCL's
    # bf16 reduction rounds a partial sum at each of up to N - 1 steps, each error within
    # 2^-8 of the partial sum, so its bound grows with the rank count (2^-7 at N = 2).
    local = out["local"]
    with np.errstate(invalid="ignore"):
        mean = local.mean(axis=0)
        bound = 2 ** -8 * max(2, WORLD) * np.abs(local).mean(axis=0) + 1e-30
        finite = np.isfinite(mean)
        assert np.array_equal(finite, np.isfinite(out["reduced"]))
        assert np.all(np.abs(out["reduced"][finite] - mean[finite]) <= bound[finite])
    if transport == "p2p":
        # The pull reduce-scatter sums in f32 in rank order and rounds once: bit-exact.
        total = local[0].astype(np.float32)
        for q in range(1, WORLD):
            total = total + local[q].astype(np.float32)
        with np.errstate(invalid="ignore"):
            expect = round_model(total * np.float32(1.0 / WORLD))
        np.testing.assert_array_equal(out["reduced"], expect)
    params = W.init_params(shape, seed=0)
    decay, no_decay = shape.groups()
    base = {"lr": 3e-4, "betas": (0.9, 0.999), "eps": 1e-8, "maximize": False}
    # Registration order of the parameters (group by group) -> original index.
    order = decay + no_decay
    oracle = oadamw.OracleAdamW(params, [(decay, {**base, "weight_decay": 0.1}),
                                         (no_decay, {**base, "weight_decay": 0.0})])
    oscaler = oamp.OracleGradScaler(1024.0, 2.0, 0.5, 2)
    shapes = [s for _, s in shape.shapes()]
    for step in range(4):
        flat = out["reduced"][step]
        grads = [None] * len(shapes)
        for k, orig in enumerate(order):   # flat-layout offsets follow the registration order
            grads[orig] = flat[offsets[k]:offsets[k] + numels[orig]].reshape(shapes[orig]).astype(np.float32).copy()
        # Eager transforms rewrite the bf16 gradient shard in place, like the reference's
        # in-place unscale_ / clip on bf16 gradient storage.
        # The device norm agrees with the oracle's two-pass norm to 1e-12; the oracle then clips
        # with the device norm, so everything after the clip compares bit for bit.
        probe = [None if g is None else g.copy() for g in grads]
        if oamp.OracleGradScaler(oscaler.scale).unscale(probe):
            if not lazy:
                probe = [None if g is None else round_model(g) for g in probe]
            ref_norm = float(oclip.total_norm([g for g in probe if g is not None], norm_type))
            assert abs(out["norms"][step] - ref_norm) <= 1e-12 * ref_norm
        r = oamp.amp_step(oracle, oscaler, grads, max_norm=1.0, norm_type=norm_type,
                          storage=None if lazy else round_model, given_norm=float(out["norms"][step]))
        assert bool(out["stepped"][step]) == r["stepped"]
    assert float(out["scale"]) == oscaler.scale
    assert out["steps"].tolist() == [3] * len(numels)
    for k, orig in enumerate(order):
        # The oracle ran on exactly the reduced gradients and the device norm: bit for bit.
        np.testing.assert_array_equal(out[f"master{k}"].view(np.uint32), params[orig].view(np.uint32))
        np.testing.assert_array_equal(out[f"m{k}"].view(np.uint32),
                                      oracle.state[orig]["exp_avg"].view(np.uint32))
        # The all-gathered model copy is the model-dtype rounding of the gathered master.
        np.testing.assert_array_equal(out[f"copy{orig}"], round_model(out[f"master{k}"]))


def _stall_worker(rank, world, port, store_port, out_path, pull="sm"):
    """Both ranks take one step; then rank 1 stops taking steps (between steps, nothing of
    it in flight) but stays alive, so its memory stays mapped, until rank 0 is done. Rank
    0's next step finds no READY from rank 1: the waits end after exchange_timeout, the
    step is skipped and the error word says so."""
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank),
                            timeout=datetime.timedelta(seconds=60))
    store = dist.TCPStore("127.0.0.1", store_port, world, rank == 0, timeout=datetime.timedelta(seconds=60))
    try:
        from namitorch_b200 import GradScaler, workloads as W
        from namitorch_b200.optim import clip_grad_norm_
        from namitorch_b200.zero import ZeroAdamW
        shape = W.CONFIG_SMALL
        params = [torch.nn.Parameter(torch.from_numpy(a).cuda()) for a in W.init_params(shape, seed=0)]
        opt = ZeroAdamW(params, lr=3e-4, model_dtype=torch.bfloat16, transport="p2p", exchange_timeout=1.0,
                        pull=pull)
        scaler = GradScaler(1024.0)

        def step():
            for p in params:
                p.grad.fill_(1.0)
            scaler.scale(torch.ones((), device="cuda"))
            scaler.unscale_(opt)
            norm = clip_grad_norm_(params, 1.0)
            stepped = scaler.step(opt)
            scaler.update()
            return norm, stepped

        step()
        torch.cuda.synchronize()
        dist.barrier()
        assert opt.exchange_error() == 0
        if rank == 0:
            before = opt.master.clone()
            norm, stepped = step()
            torch.cuda.synchronize()
            error = opt.exchange_error()
            try:
                opt.check_exchange()
                raised = ""
            except RuntimeError as exc:
                raised = str(exc)
            np.savez(out_path, error=error, stepped=bool(stepped), norm=float(norm.item()),
                     unchanged=bool(torch.equal(before, opt.master)), raised=raised)
            store.set("done", "1")
        else:
            store.wait(["done"])
        opt.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("pull", ["sm", "copy"])
def test_a_rank_that_stops_between_steps_makes_the_others_skip_with_an_error(tmp_path, pull):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    out_path = tmp_path / "stall.npz"
    mp.spawn(_stall_worker, args=(2, _free_port(), _free_port(), str(out_path), pull), nprocs=2, join=True)
    out = np.load(out_path)
    assert int(out["error"]) == 3          # the reduce-scatter's wait and the update's wait both ran out
    assert not bool(out["stepped"]) and np.isnan(float(out["norm"]))
    assert bool(out["unchanged"])          # the skipped step left the master weights alone
    assert "wait on another rank ran out" in str(out["raised"])
