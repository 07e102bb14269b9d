"""The checker bench.py runs after its timed region (the reference's own AdamW from the
baseline/_ref install, fed the unscaled and clipped gradient) agrees with the oracle's
restatement bit for bit, with and without a prior state and for both weight-decay groups.
Skipped when the reference install is absent."""
import numpy as np
import pytest

from conftest import REPO

import bench
from oracle import adamw as oadamw


@pytest.fixture(scope="module")
def reference_install():
    if bench.load_reference_package() is None:
        pytest.skip("baseline/_ref (the reference install) is not present")


@pytest.mark.parametrize("step_count,wd,norm", [(0, 0.1, 3.5), (7, 0.0, 0.25), (40, 0.1, 1.0 - 1e-6)])
def test_shard_checker_matches_oracle(reference_install, step_count, wd, norm):
    rng = np.random.default_rng(step_count)
    n = 4099
    pre = [rng.normal(0, 0.02, n).astype(np.float32), rng.normal(0, 1e-3, n).astype(np.float32),
           np.abs(rng.normal(0, 1e-6, n)).astype(np.float32)]
    if step_count == 0:
        pre[1][:] = 0
        pre[2][:] = 0
    reduced = (rng.normal(0, 1e-3, n) * 65536).astype(np.float32)
    group = {"lr": 3e-4, "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay": wd}
    got, checker = bench._shard_reference(pre, reduced, 65536.0, norm, step_count, group, True, "cpu")
    assert checker.startswith("reference AdamW")
    g = (reduced / np.float32(65536.0)).astype(np.float32)
    coef = 1.0 / (norm + 1e-6)
    if coef < 1:
        g = (g.astype(np.float64) * coef).astype(np.float32)
    p, m, v = (a.copy() for a in pre)
    oadamw.adam_update(p, g, m, v, step_count, lr=3e-4, beta1=0.9, beta2=0.999, eps=1e-8, weight_decay=wd)
    for ours, want in zip(got, (p, m, v)):
        np.testing.assert_array_equal(np.asarray(ours).view(np.uint32), want.view(np.uint32))


def test_skipped_step_expects_the_state_unchanged(reference_install):
    pre = [np.arange(5, dtype=np.float32)] * 3
    got, checker = bench._shard_reference(pre, np.ones(5, np.float32), 2.0, 1.0, 3, {}, False, "cpu")
    assert checker.startswith("skipped") and all(np.array_equal(a, b) for a, b in zip(got, pre))


def test_reference_arm_runs_the_reference_on_the_shared_sample(reference_install):
    """The reference arm's CPU figure comes from the reference's own AMP step on the same
    16.8M-parameter sample as the threaded port beside it."""
    assert bench.CPU_SAMPLE_PARAMS == 16_789_504
    ref = bench.reference_amp_sample(steps=1, warmup=0)
    assert ref["kind"] == "reference" and ref["cores"] == 1 and ref["value"] > 0
    assert str(bench.CPU_SAMPLE_PARAMS) in ref["sample"] and ref["host"]["cpu_count"] >= 1
    port = bench.cpu_amp_sample(1, 2, warmup=0)
    assert port["kind"] == "port" and port["cores"] == 2 and str(bench.CPU_SAMPLE_PARAMS) in port["sample"]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_zero_parity_checks_the_group_the_optimizer_registered(world):
    """ZeroAdamW indexes its pieces in registration order (the decay group's parameters,
    then the no-decay group's), which is not the model's order. The slice the multi-GPU
    self-check takes must be looked up in that order, or its weight decay comes from the
    wrong group; at N = 4 and 8 on the 1.3B layout some ranks' largest piece is such a
    parameter, and the check then reported every master element of those ranks wrong."""
    from types import SimpleNamespace
    from namitorch_b200 import workloads as W
    from namitorch_b200.zero import interleaved_layout, owned_ranges, shard_pieces
    shape = W.CONFIG_1P3B
    numel = [int(np.prod(s)) for _, s in shape.shapes()]
    decay, no_decay = shape.groups()
    order = decay + no_decay
    model = [SimpleNamespace(index=k) for k in range(len(numel))]
    registered = [model[k] for k in order]
    numels = [numel[k] for k in order]
    offsets, total, c = interleaved_layout(numels, world, 1)
    differs = 0
    for rank in range(world):
        opt = SimpleNamespace(pieces=shard_pieces(offsets, numels, owned_ranges(world, rank, 1, c)),
                              params_list=registered)
        i, off, n, prm = bench.parity_piece(opt)
        assert n > 0 and prm is registered[i]
        assert (prm.index in decay) == (i < len(decay))
        differs += (i in decay) != (prm.index in decay)   # model order would pick the other group
    assert differs == {2: 0, 4: 2, 8: 3}[world]


def test_nvlink_floor_arithmetic(monkeypatch):
    """The ZeRO-1 floors of the N > 1 line from given link rates: each phase moves
    (N - 1)/N x 2 B per parameter per GPU and direction; the update phase's floor is the
    longer of its link time and its HBM time (28 B per shard parameter plus the peers'
    incoming 2 B copies), so it is HBM-bound at N = 2 and link-bound at N = 8."""
    from types import SimpleNamespace
    monkeypatch.setattr(bench, "measure_peer_bandwidth", lambda world, rank, device: {"pull_gbs": 640.0,
                                                                                       "push_gbs": 630.0})
    monkeypatch.setattr(bench, "measured_peak", lambda: (6500.0, "measured"))
    P = 1_315_721_216
    for world, bound in ((2, "hbm"), (8, "nvlink")):
        link = 2.0 * P * (world - 1) / world
        out = bench.nvlink_section(SimpleNamespace(rank=0, device="cpu"), P, world, 7.0,
                                   {"reduce_scatter": 3.0, "update_with_overlapped_all_gather": 3.5})
        assert out["bytes_per_gpu_per_phase"] == link
        assert abs(out["floor_ms"] - (link / 640e9 + link / 630e9) * 1e3) < 1e-9
        hbm_update = (bench.BYTES_UPDATE + 2.0 * (world - 1)) * (P / world) / 6500e9 * 1e3
        assert abs(out["update_phase"]["floor_ms"] - max(link / 630e9 * 1e3, hbm_update)) < 1e-9
        assert out["update_phase"]["bound"] == bound
        assert abs(out["reduce_scatter_gbs"] - link / 3.0e-3 / 1e9) < 1e-6
