"""Fleet planning on the GPU: per-vehicle masses in the learned scorer against
the oracle, and candidate-range shards (lwm_planner_set_shard /
lwm_plan_device_shard / lwm_mppi_combine_device) against the unsharded
planner.  The shards run one after another on one GPU here; across GPUs the
only difference is that fleet.exchange_tuples gathers the tuples over NCCL."""
import dataclasses

import numpy as np
import pytest

import lewm_b200 as L
import oracle as O
from gpu_helpers import assert_actions_close, assert_costs_close, assert_same_argmin, normals
from lewm_b200 import fleet as F
from lewm_b200 import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _norm(w):
    return (w.state_mean, w.state_std, w.action_mean, w.action_std)


def _sky(ctx, w, masses=None):
    sc = L.SkyJepaScorer(ctx, w.model, w.weights, w.state_mean, w.state_std, w.action_mean, w.action_std, w.cost,
                         w.dt)
    sc.set_context(w.state_history, w.action_history, w.reference_states, w.reference_actions, vehicle_mass=masses)
    return sc


def _nominal(ctx, w):
    sc = L.NominalScorer(ctx, w.dt, w.trim, w.cost, w.substeps)
    sc.set_context(w.initial, w.motors, w.reference_states, w.reference_actions)
    return sc


def test_vehicle_masses_match_oracle(ctx):
    w = W.fleet(seed=4, vehicles=3, samples=96, horizon=12)
    cand = (w.hover + normals(41, (3, 96, 12, 4)) * 0.6).astype(np.float32)
    sc = _sky(ctx, w, w.masses)
    d = torch.as_tensor(cand).cuda()
    out = torch.empty((3, 96), device="cuda")
    torch.cuda.synchronize()
    sc.score_device(d.data_ptr(), 3, 96, 12, 4, out.data_ptr())
    ctx.synchronize()
    m = O.SkyJepaModel(w.model, w.weights)
    ref = m.scores(_norm(w), w.state_history, w.action_history, w.reference_states, w.reference_actions, w.cost,
                   w.dt, cand, masses=w.masses)
    assert_costs_close(out.cpu().numpy(), ref)
    # the masses matter: the default mass gives other costs
    ref_default = m.scores(_norm(w), w.state_history, w.action_history, w.reference_states, w.reference_actions,
                           w.cost, w.dt, cand)
    assert np.abs(ref_default - ref).max() > 1e-3 * np.abs(ref).max()


def test_fleet_mppi_with_masses_matches_oracle(ctx):
    w = W.fleet(seed=5, vehicles=2, samples=128, horizon=10)
    noise = normals(43, (1, 2, 128, 10, 4))
    p = L.MppiPlanner(ctx, w.mppi)
    r = p.plan(_sky(ctx, w, w.masses), injected_noise=noise)
    m = O.SkyJepaModel(w.model, w.weights)
    c = m.score_ctx(_norm(w), w.state_history, w.action_history, w.reference_states, w.reference_actions, w.cost,
                    w.dt, masses=w.masses)
    ref = O.mppi_plan(w.mppi, 2, (O.SKYJEPA_FN, c), noise=noise)
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"])
    assert_same_argmin(r.best_indices, ref["best"], ref["scores"])


def _sharded(ctx, make_scorer, cfg, shards, warm):
    """Plan with `shards` candidate shards on one GPU; returns (sequence,
    best indices, warm start)."""
    planners, tuples = [], []
    for i in range(shards):
        s0, s1 = F.split_range(cfg.samples, shards, i)
        p = L.MppiPlanner(ctx, dataclasses.replace(cfg, samples=s1 - s0))
        p.set_shard(s0, cfg.samples)
        p.set_warm_start_sequence(warm)
        sc = make_scorer()
        ptr, width = p.plan_device_shard(sc)
        ctx.synchronize()
        tuples.append(L.device_tensor(ptr, (sc.batch, width)).clone())
        planners.append(p)
    gathered = torch.stack(tuples).contiguous()
    ctx.synchronize()
    res = planners[0].combine_device(gathered.data_ptr(), shards)
    ctx.synchronize()
    B, T, A = res.batch, cfg.horizon, cfg.action_dim
    seq = L.device_tensor(res.sequence, (B, T, A)).cpu().numpy()
    best = L.device_tensor(res.best_indices, (B,), "u4").cpu().numpy()
    warm = planners[0].warm_start_sequence()
    return seq, best, warm


@pytest.mark.parametrize("shards", [2, 3])
def test_nominal_candidate_shards_equal_unsharded(ctx, shards):
    w = W.nominal(seed=6, batch=2, samples=512, horizon=15)
    full = L.MppiPlanner(ctx, w.mppi)
    full.set_warm_start_sequence(w.warm_start)
    ref = full.plan(_nominal(ctx, w))
    seq, best, warm = _sharded(ctx, lambda: _nominal(ctx, w), w.mppi, shards, w.warm_start)
    assert_actions_close(seq, ref.sequence)
    assert_same_argmin(best, ref.best_indices, ref.scores)
    np.testing.assert_allclose(warm, full.warm_start_sequence(), atol=1e-4)


def test_skyjepa_candidate_shards_equal_unsharded(ctx):
    w = W.fleet(seed=7, vehicles=2, samples=256, horizon=10)
    full = L.MppiPlanner(ctx, w.mppi)
    full.set_warm_start_sequence(w.warm_start)
    ref = full.plan(_sky(ctx, w, w.masses))
    seq, best, _ = _sharded(ctx, lambda: _sky(ctx, w, w.masses), w.mppi, 2, w.warm_start)
    assert_actions_close(seq, ref.sequence)
    assert_same_argmin(best, ref.best_indices, ref.scores)


def test_shard_validation(ctx):
    w = W.nominal(seed=8, samples=64)
    p = L.MppiPlanner(ctx, w.mppi)
    with pytest.raises(L.LwmError, match="exceed sample_total"):
        p.set_shard(10, 64)
    p.set_shard(0, 128)
    with pytest.raises(L.LwmError, match="candidate shard"):
        p.plan(_nominal(ctx, w))
    p.set_shard(0, 0)
    p.plan(_nominal(ctx, w))


def test_fleet_planner_single_rank(ctx):
    w = W.fleet(seed=9, vehicles=3, samples=200, horizon=8)
    part = F.partition(3, 200, 1)[0]
    fp = F.FleetPlanner(ctx, part, _sky(ctx, w, w.masses), w.mppi)
    res = fp.plan_device()
    ctx.synchronize()
    ref = L.MppiPlanner(ctx, w.mppi).plan(_sky(ctx, w, w.masses))
    seq = L.device_tensor(res.sequence, (3, 8, 4)).cpu().numpy()
    assert_actions_close(seq, ref.sequence)
