"""ZeRO-1 host logic on CPU ranks (gloo, world size 2).

The collective choreography of ``namitorch_b200.zero.ZeroAdamW`` — shard layout,
reduce-scatter of the gradient buffer, the statistics all-reduce that makes every rank take
the same clip decision, the all-gather of the model copy and the state_dict gather — runs
here on CPU processes. ``NumpyShardKernels`` is a test double for the CUDA kernel calls:
it applies the same float32 operation sequence with NumPy (the product itself has no CPU
path; without this double ZeroAdamW refuses CPU tensors). The result is checked against
the single-process oracle fed with the summed gradients.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from namitorch_b200 import _native as N
from namitorch_b200.flat import SEGMENT_DTYPE
from namitorch_b200.zero import interleaved_layout, owned_ranges, shard_pieces

SIZES = [(37, 5), (100,), (1000,), (7,), (64, 64), (3,)]


def test_shard_partition_covers_every_element_once():
    numels = [int(np.prod(s)) for s in SIZES]
    for world in (1, 2, 3, 4, 8):
        for pieces in (1, 3, 8):
            offsets, total, c = interleaved_layout(numels, world, pieces)
            assert total == pieces * world * c and c % 64 == 0
            covered = np.zeros(total, np.int32)
            for rank in range(world):
                ranges = owned_ranges(world, rank, pieces, c)
                assert [r[2] for r in ranges] == [j * c for j in range(pieces)]
                for i, off, n, j in shard_pieces(offsets, numels, ranges):
                    start, stop, local = ranges[j]
                    lo = start + off - local
                    assert offsets[i] <= lo and lo + n <= offsets[i] + numels[i] and lo + n <= stop
                    covered[lo:lo + n] += 1
            for off, n in zip(offsets, numels):
                assert np.all(covered[off:off + n] == 1)


class NumpyShardKernels:
    """Test double of zero.CudaShardKernels (float32 NumPy, same operation order)."""

    def __init__(self):
        self.opt = None

    @staticmethod
    def _values(buf, scale):
        g = buf.detach().float().numpy().copy()
        if scale is not None:
            g = g / np.float32(scale.item())
        return g

    def stats(self, buf, stats, *, scale, norm_type, pass_, finalize):
        g = self._values(buf, scale)
        s = stats.numpy()
        if pass_ == 0:
            finite = np.isfinite(g)
            s[0] = float(np.sum(np.square(g[finite].astype(np.float64))))
            s[1] = float(np.count_nonzero(~finite))
            s[2] = float(np.count_nonzero(np.isnan(g)))
            s[3] = float(np.max(np.abs(g[~np.isnan(g)]), initial=0.0))
        else:
            s[4] = float(np.sum(np.power(np.abs(g.astype(np.float64)) / s[3], norm_type)))
        if finalize:
            self.finalize(stats, norm_type)

    @staticmethod
    def finalize(stats, norm_type):
        s = stats.numpy()
        s[6] = 1.0 if s[1] > 0 else 0.0
        if s[2] > 0:
            s[5] = np.nan
        elif s[1] > 0:
            s[5] = np.inf
        elif s[3] == 0:
            s[5] = 0.0
        elif np.isinf(norm_type):
            s[5] = s[3]
        elif norm_type == 2.0:
            s[5] = np.sqrt(s[0])
        else:
            s[5] = s[3] * s[4] ** (1.0 / norm_type)

    def transform(self, buf, *, scale, stats, max_norm):
        g = self._values(buf, scale)
        if max_norm is not None:
            coef = max_norm / (stats[5].item() + 1e-6)
            if coef < 1:
                g = (g.astype(np.float64) * coef).astype(np.float32)
        buf.copy_(torch.from_numpy(g))

    def clip_value(self, buf, bound):
        g = buf.detach().numpy().astype(np.float64)
        buf.copy_(torch.from_numpy(np.clip(g, -bound, bound).astype(np.float32)))

    def update(self, *, master, exp_avg, exp_avg_sq, copy, grad_dtype, segments, num_segments, num_chunks, steps,
               corrections, capacity, scale, stats, skip, max_norm, groups, peers=None):
        assert not peers   # the CPU ranks use the collective transport
        s = None if stats is None else stats.numpy()
        if skip and s[6] != 0:
            return
        coef = None
        if max_norm is not None:
            c = max_norm / (s[5] + 1e-6)
            coef = c if c < 1 else None
        table = np.frombuffer(segments.numpy().tobytes(), SEGMENT_DTYPE)
        gshard = self._values(self.opt.grad_shard, scale)
        p, m, v = master.numpy(), exp_avg.numpy(), exp_avg_sq.numpy()
        corr = corrections.numpy()
        st = steps.numpy()
        f32 = np.float32
        for seg in table:
            off, n, gi, slot = int(seg["offset"]), int(seg["count"]), int(seg["group"]), int(seg["step_slot"])
            gr = groups[gi]
            g = gshard[off:off + n]
            if coef is not None:
                g = (g.astype(np.float64) * coef).astype(np.float32)
            t = min(int(st[slot if slot >= 0 else -slot - 1]) + 1, capacity - 1)
            c1, c2 = corr[gr.correction_row, t]
            pp, mm, vv = p[off:off + n], m[off:off + n], v[off:off + n]
            mm[...] = f32(gr.beta1) * mm + f32(gr.one_minus_beta1) * g
            vv[...] = f32(gr.beta2) * vv + f32(gr.one_minus_beta2) * g * g
            u = (mm / c1) / (np.sqrt(vv / c2) + f32(gr.eps))
            if gr.update_parameter:
                base = pp * f32(gr.decay_factor) if gr.decay_mode == N.NT_DECAY_DECOUPLED else pp
                pp[...] = base - f32(gr.lr) * u
            if slot >= 0:   # a negative slot is advanced by the parameter's last piece
                st[slot] += 1
            copy[off:off + n].copy_(master[off:off + n].to(copy.dtype))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_grads(rank, step):
    rng = np.random.default_rng(100 * step + rank)
    return [rng.normal(0, 0.3, s).astype(np.float32) for s in SIZES]


CLIP_VALUE_STEP = 1   # the step that also applies clip_grad_value_(0.5) after the norm clip


def _worker(rank, world, port, result_path, lazy):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from namitorch_b200.optim import clip_grad_norm_, clip_grad_value_, defer_gradient_transforms, get_grad_norm
        from namitorch_b200.zero import ZeroAdamW
        defer_gradient_transforms(lazy)
        rng = np.random.default_rng(0)
        arrays = [rng.normal(0, 1, s).astype(np.float32) for s in SIZES]
        params = [torch.nn.Parameter(torch.from_numpy(a.copy())) for a in arrays]
        kernels = NumpyShardKernels()
        groups = [{"params": [params[i] for i in (0, 2, 4)], "weight_decay": 0.1},
                  {"params": [params[i] for i in (1, 3, 5)], "weight_decay": 0.0}]
        opt = ZeroAdamW(groups, lr=1e-2, model_dtype=torch.float32, average_grads=False, _kernels=kernels)
        kernels.opt = opt
        norms = []
        for step in range(3):
            opt.zero_grad()
            for p, g in zip(params, _rank_grads(rank, step)):
                p.grad.copy_(torch.from_numpy(g))
            before = float(get_grad_norm(params).item())   # the global norm of the reduced gradients
            norms.append(float(clip_grad_norm_(params, 5.0).item()))
            assert abs(before - norms[-1]) <= 1e-12 * norms[-1]
            if step == CLIP_VALUE_STEP:
                clip_grad_value_(params, 0.5)
            opt.step()
        sd = opt.state_dict()
        copies = [p.detach().numpy().copy() for p in params]
        order = [0, 2, 4, 1, 3, 5]   # registration order: group by group
        # Round trip: a fresh optimizer loaded from the gathered state takes the same 4th step.
        params2 = [torch.nn.Parameter(torch.from_numpy(a.copy())) for a in arrays]
        kernels2 = NumpyShardKernels()
        groups2 = [{"params": [params2[i] for i in (0, 2, 4)], "weight_decay": 0.1},
                   {"params": [params2[i] for i in (1, 3, 5)], "weight_decay": 0.0}]
        opt2 = ZeroAdamW(groups2, lr=1e-2, model_dtype=torch.float32, average_grads=False, _kernels=kernels2)
        kernels2.opt = opt2
        opt2.load_state_dict(sd)
        for k in range(len(params)):
            np.testing.assert_array_equal(params2[k].detach().numpy(), copies[k])
        for o, ps in ((opt, params), (opt2, params2)):
            o.zero_grad()
            for p, g in zip(ps, _rank_grads(rank, 3)):
                p.grad.copy_(torch.from_numpy(g))
            o.step()
        sd_a, sd_b = opt.state_dict(), opt2.state_dict()
        for k in sd_a["state"]:
            assert sd_a["state"][k]["step"] == sd_b["state"][k]["step"] == 4
            for name in ("exp_avg", "exp_avg_sq", "master_param"):
                np.testing.assert_array_equal(sd_a["state"][k][name].numpy(), sd_b["state"][k][name].numpy())
        for k in range(len(params)):
            np.testing.assert_array_equal(params2[k].detach().numpy(), params[k].detach().numpy())
        if rank == 0:
            np.savez(result_path, norms=np.array(norms),
                     **{f"master{order[k]}": sd["state"][k]["master_param"].numpy() for k in sd["state"]},
                     **{f"m{order[k]}": sd["state"][k]["exp_avg"].numpy() for k in sd["state"]},
                     **{f"copy{k}": copies[k] for k in range(len(copies))},
                     steps=np.array([sd["state"][k]["step"] for k in sorted(sd["state"])]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("lazy", [True, False], ids=["deferred", "eager"])
def test_zero1_two_ranks_match_single_process_oracle(tmp_path, lazy):
    from oracle import adamw as oadamw
    from oracle import clip as oclip
    result = tmp_path / "zero.npz"
    mp.spawn(_worker, args=(2, _free_port(), str(result), lazy), nprocs=2, join=True)
    out = np.load(result)
    rng = np.random.default_rng(0)
    arrays = [rng.normal(0, 1, s).astype(np.float32) for s in SIZES]
    base = {"lr": 1e-2, "betas": (0.9, 0.999), "eps": 1e-8, "maximize": False}
    oracle = oadamw.OracleAdamW(arrays, [([0, 2, 4], {**base, "weight_decay": 0.1}),
                                         ([1, 3, 5], {**base, "weight_decay": 0.0})])
    for step in range(3):
        grads = [a + b for a, b in zip(_rank_grads(0, step), _rank_grads(1, step))]
        norm = oclip.clip_grad_norm_(grads, 5.0)
        assert abs(out["norms"][step] - float(norm)) <= 1e-12 * float(norm)
        if step == CLIP_VALUE_STEP:
            oclip.clip_grad_value_(grads, 0.5)
        oracle.step(grads)
    assert out["steps"].tolist() == [3] * len(SIZES)
    # (the summed norm differs from the reference's two-pass norm in the last bits, so the
    # clip coefficient can differ by an ulp: compare to 1e-6)
    for k in range(len(SIZES)):
        np.testing.assert_allclose(out[f"master{k}"], arrays[k], rtol=1e-6, atol=1e-9)
        np.testing.assert_allclose(out[f"m{k}"], oracle.state[k]["exp_avg"], rtol=1e-6, atol=1e-9)
        np.testing.assert_array_equal(out[f"copy{k}"], out[f"master{k}"])


@pytest.mark.parametrize("kwargs,match", [
    ({"transport": "tcp"}, "transport"), ({"exchange": "mpi"}, "exchange"), ({"pull": "dma"}, "pull"),
    ({"pull": "copy", "exchange": "nccl"}, "exchange='flags'"), ({"exchange_timeout": 0}, "exchange_timeout"),
    ({"pieces": 0}, "pieces"), ({"model_dtype": torch.int8}, "model_dtype")])
def test_zero_adamw_rejects_bad_options_before_any_collective(kwargs, match):
    """Option checks come first, so a bad option raises on every rank alike and no rank is
    left inside a collective."""
    from namitorch_b200.zero import ZeroAdamW
    params = [torch.nn.Parameter(torch.zeros(4))]
    with pytest.raises((ValueError, TypeError), match=match):
        ZeroAdamW(params, **kwargs)
