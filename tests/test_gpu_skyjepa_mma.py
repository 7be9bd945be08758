"""The f32 learned SkyJEPA scorer on the tensor cores with split-fp16
operands (every GEMM operand as two fp16 halves, three partial products per
product, f32 accumulation, gates and tail) against the f32 oracle at the f32
tolerances: per-candidate costs within 1e-4 relative, the MPPI sequence
within 1e-4, the best index up to ties — several vehicles with their own
masses, horizons that are odd and long, more 128-row clusters than one wave,
the seeded Philox path, and agreement with the CUDA-core f32 rollout."""
import dataclasses

import numpy as np
import pytest

import lewm_b200 as L
import oracle as O
from gpu_helpers import assert_actions_close, assert_costs_close, assert_same_argmin, normals
from lewm_b200 import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _norm(w):
    return (w.state_mean, w.state_std, w.action_mean, w.action_std)


def _scorer(ctx, w, masses=None, precision="f32"):
    sc = L.SkyJepaScorer(ctx, w.model, w.weights, w.state_mean, w.state_std, w.action_mean, w.action_std, w.cost,
                         w.dt)
    sc.set_precision(precision)
    sc.set_context(w.state_history, w.action_history, w.reference_states, w.reference_actions, vehicle_mass=masses)
    return sc


def _oracle_plan(w, noise, masses=None):
    m = O.SkyJepaModel(w.model, w.weights)
    c = m.score_ctx(_norm(w), w.state_history, w.action_history, w.reference_states, w.reference_actions, w.cost,
                    w.dt, masses=masses)
    return O.mppi_plan(w.mppi, w.batch, (O.SKYJEPA_FN, c), noise=noise, warm_start=w.warm_start)


def _plan(ctx, w, noise, masses=None):
    p = L.MppiPlanner(ctx, w.mppi)
    p.set_warm_start_sequence(w.warm_start)
    sc = _scorer(ctx, w, masses)
    n0 = ctx.launch_count()
    r = p.plan(sc, injected_noise=noise)
    assert ctx.launch_count() - n0 == 3, "the split-fp16 tensor-core path was not taken"
    return r, p, sc


@pytest.mark.parametrize("batch, samples, horizon", [(1, 512, 15), (2, 256, 7), (1, 128, 30), (1, 128, 1), (1, 256, 2)])
def test_split_fp16_mppi_matches_oracle(ctx, batch, samples, horizon):
    w = W.skyjepa(seed=51, batch=batch, samples=samples, horizon=horizon)
    noise = normals(81, (1, batch, samples, horizon, 4))
    r, _, _ = _plan(ctx, w, noise)
    ref = _oracle_plan(w, noise)
    rel = np.abs(np.asarray(r.scores, np.float64) - ref["scores"]) / np.maximum(np.abs(ref["scores"]), 1e-6)
    print(f"split-fp16 vs f32 oracle: worst {rel.max():.3e}, mean {rel.mean():.3e}, cost range {ref['scores'].min():.4g}..{ref['scores'].max():.4g}")
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"])
    assert_same_argmin(r.best_indices, ref["best"], ref["scores"])


def test_split_fp16_fleet_with_masses_and_more_clusters_than_a_wave(ctx):
    # 24 vehicles x 1024 candidates = 192 clusters of 16 CTAs (several waves)
    w = W.fleet(seed=52, vehicles=24, samples=1024, horizon=9)
    noise = normals(82, (1, 24, 1024, 9, 4))
    r, p, sc = _plan(ctx, w, noise, w.masses)
    ref = _oracle_plan(w, noise, w.masses)
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"])
    assert_same_argmin(r.best_indices, ref["best"], ref["scores"])
    # a second plan from the warm start it left (fresh barriers, cleared arrival counters)
    w.warm_start = p.warm_start_sequence()
    noise2 = normals(83, (1, 24, 1024, 9, 4))
    r2 = p.plan(sc, injected_noise=noise2)
    ref2 = _oracle_plan(w, noise2, w.masses)
    assert_costs_close(r2.scores, ref2["scores"])
    assert_actions_close(r2.sequence, ref2["sequence"])


def test_split_fp16_seeded_plan_matches_cuda_core_rollout(ctx):
    w = W.skyjepa(seed=53, batch=2, samples=384, horizon=12)
    res = {}
    for prec in ("f32", "f32-cuda-core"):
        p = L.MppiPlanner(ctx, w.mppi)
        p.set_warm_start_sequence(w.warm_start)
        res[prec] = p.plan(_scorer(ctx, w, precision=prec))
    assert_costs_close(res["f32"].scores, res["f32-cuda-core"].scores)
    assert_actions_close(res["f32"].sequence, res["f32-cuda-core"].sequence)


def test_split_fp16_context_changes_between_back_to_back_plans(ctx):
    # One scorer and planner, the context replaced between plans that run back
    # to back on one stream: the history encoder, the input kernel and the
    # rollout are chained by programmatic dependent launch, and each plan must
    # read the h0 and x tiles of its own context (not the previous plan's).
    wa = W.skyjepa(seed=53, batch=2, samples=256, horizon=8)
    other = W.skyjepa(seed=54, batch=2, samples=256, horizon=8)
    # the same model, weights and normalisation; another state / action
    # history and reference window
    wb = dataclasses.replace(wa, state_history=other.state_history, action_history=other.action_history,
                             reference_states=other.reference_states, reference_actions=other.reference_actions,
                             initial=other.initial)
    noise = normals(84, (1, 2, 256, 8, 4))
    p = L.MppiPlanner(ctx, wa.mppi)
    sc = _scorer(ctx, wa)
    for w in (wa, wb, wa):
        sc.set_context(w.state_history, w.action_history, w.reference_states, w.reference_actions)
        p.set_warm_start_sequence(w.warm_start)
        r = p.plan(sc, injected_noise=noise)
        ref = _oracle_plan(w, noise)
        assert_costs_close(r.scores, ref["scores"])
        assert_actions_close(r.sequence, ref["sequence"])
