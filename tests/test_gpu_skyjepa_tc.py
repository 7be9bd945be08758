"""Learned SkyJEPA MPPI on the tcgen05 tensor cores (bf16 weights and
recurrent state, f32 accumulation) against the f32 oracle: per-candidate
costs within 2e-2 relative (the bf16 predictor tolerance), the MPPI sequence
close to the oracle's, and the tensor-core path actually taken (it launches
four kernels per iteration: sampling, per-step inputs, h0 and the persistent rollout)."""
import numpy as np
import pytest

import lewm_b200 as L
import oracle as O
from gpu_helpers import normals
from lewm_b200 import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

BF16_REL = 2e-2


def _norm(w):
    return (w.state_mean, w.state_std, w.action_mean, w.action_std)


def _scorer(ctx, w, masses=None, precision="bf16"):
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


def _check(r, ref):
    s, rs = np.asarray(r.scores, np.float64), np.asarray(ref["scores"], np.float64)
    rel = np.abs(s - rs) / np.maximum(np.abs(rs), 1e-6)
    assert rel.max() <= BF16_REL, f"worst relative cost error {rel.max():.3e}"
    # the weighted sequence: a convex combination of candidates whose weights
    # carry the cost error; compare against the spread of the candidates
    scale = np.abs(ref["sequence"]).max()
    assert np.abs(np.asarray(r.sequence) - ref["sequence"]).max() <= 5e-2 * scale


@pytest.mark.parametrize("batch, samples, horizon", [(1, 512, 15), (2, 256, 10)])
def test_tc_mppi_matches_oracle(ctx, batch, samples, horizon):
    w = W.skyjepa(seed=21, batch=batch, samples=samples, horizon=horizon)
    noise = normals(61, (1, batch, samples, horizon, 4))
    p = L.MppiPlanner(ctx, w.mppi)
    p.set_warm_start_sequence(w.warm_start)
    sc = _scorer(ctx, w)
    n0 = ctx.launch_count()
    r = p.plan(sc, injected_noise=noise)
    assert ctx.launch_count() - n0 == 4, "the tensor-core path was not taken"
    _check(r, _oracle_plan(w, noise))


def test_tc_fleet_with_masses_matches_oracle(ctx):
    w = W.fleet(seed=22, vehicles=3, samples=384, horizon=30)
    noise = normals(62, (1, 3, 384, 30, 4))
    p = L.MppiPlanner(ctx, w.mppi)
    p.set_warm_start_sequence(w.warm_start)
    r = p.plan(_scorer(ctx, w, w.masses), injected_noise=noise)
    _check(r, _oracle_plan(w, noise, w.masses))


def test_tc_seeded_plan_matches_f32_path(ctx):
    # the same Philox candidates on both paths: scores agree within the bf16 tolerance
    w = W.skyjepa(seed=23, batch=2, samples=256, horizon=12)
    res = {}
    for prec in ("f32", "bf16"):
        p = L.MppiPlanner(ctx, w.mppi)
        p.set_warm_start_sequence(w.warm_start)
        res[prec] = p.plan(_scorer(ctx, w, precision=prec))
    s32, s16 = np.asarray(res["f32"].scores, np.float64), np.asarray(res["bf16"].scores, np.float64)
    assert (np.abs(s16 - s32) / np.maximum(np.abs(s32), 1e-6)).max() <= BF16_REL


def test_tc_unsupported_shape_keeps_f32(ctx):
    w = W.skyjepa(seed=24, samples=100, horizon=8)   # 100 is not a multiple of 128
    p = L.MppiPlanner(ctx, w.mppi)
    n0 = ctx.launch_count()
    p.plan(_scorer(ctx, w))
    assert ctx.launch_count() - n0 == 1
