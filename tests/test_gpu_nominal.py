"""Fused nominal-physics MPPI on the GPU against the oracle (the reference's
CPU plant path, src/models/skyjepa/nominal.rs:50-71 + control.rs:430-452)."""
import numpy as np
import pytest

import lewm_b200 as L
import oracle as O
from gpu_helpers import assert_actions_close, assert_costs_close, assert_same_argmin, normals
from lewm_b200 import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _scorer(ctx, w, domains=None):
    sc = L.NominalScorer(ctx, w.dt, w.trim, w.cost, w.substeps)
    sc.set_context(w.initial, w.motors, w.reference_states, w.reference_actions, domains)
    return sc


def _oracle_fn(w, domains=None):
    c = O.nominal_ctx(w.initial, w.motors, w.reference_states, w.reference_actions, w.cost, w.dt, w.trim,
                      w.substeps, domains=domains)
    return (O.NOMINAL_FN, c)


def test_nominal_mppi_matches_oracle_injected_noise(ctx):
    w = W.nominal(seed=1)
    noise = normals(100, (1, 1, 512, 15, 4))
    p = L.MppiPlanner(ctx, w.mppi)
    p.set_warm_start_sequence(w.warm_start)
    r = p.plan(_scorer(ctx, w), injected_noise=noise)
    ref = O.mppi_plan(w.mppi, 1, _oracle_fn(w), noise=noise, warm_start=w.warm_start)
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"])
    assert_same_argmin(r.best_indices, ref["best"], ref["scores"])
    assert_actions_close(p.warm_start_sequence(), ref["warm"])


def test_nominal_mppi_seeded_matches_oracle_philox(ctx):
    w = W.nominal(seed=2)
    p = L.MppiPlanner(ctx, w.mppi)
    p.set_warm_start_sequence(w.warm_start)
    r = p.plan(_scorer(ctx, w))
    ref = O.mppi_plan(w.mppi, 1, _oracle_fn(w), seed=w.mppi.seed, offset=0, warm_start=w.warm_start)
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"])


def test_nominal_predicted_states_match_cpu_plant(ctx):
    # tests/skyjepa_nominal.rs:8-51 bound is 2e-3; the GPU follows the plant's
    # operation order, so the states agree far more tightly.
    w = W.nominal(seed=3, samples=64)
    cand = (w.hover + normals(5, (1, 64, 15, 4)) * 0.5).astype(np.float32)
    sc = _scorer(ctx, w)
    d = torch.as_tensor(cand).cuda()
    states = torch.empty((1, 64, 15, 18), device="cuda")
    torch.cuda.synchronize()
    sc.predict_device(d.data_ptr(), 1, 64, 15, states.data_ptr())
    ctx.synchronize()
    _, ref_states = O.nominal_scores(w.initial, w.motors, w.reference_states, w.reference_actions, w.cost, w.dt,
                                     w.trim, cand, with_states=True)
    assert np.abs(states.cpu().numpy() - ref_states).max() < 1e-4


@pytest.mark.parametrize("trim", [1.0, 2.0])
def test_nominal_scorer_hover_cost_and_ordering(ctx, trim):
    # tests/skyjepa_nominal.rs:84-115 on the GPU path
    d = L.Domain.default()
    hover = np.float32(d.mass * d.gravity / 4.0)
    s = L.hover_state()
    T = 15
    sc = L.NominalScorer(ctx, 0.05, trim, L.TrackingCost.paper())
    sc.set_context(s[None], np.full((1, 4), hover, np.float32), np.tile(s, (1, T, 1)),
                   np.full((1, T, 4), hover * trim, np.float32))
    cand = np.concatenate([np.full((1, 1, T, 4), hover * trim + dlt, np.float32) for dlt in (0.5, 0.0, -0.5)], 1)
    dc = torch.as_tensor(cand).cuda()
    out = torch.empty((1, 3), device="cuda")
    torch.cuda.synchronize()
    sc.score_device(dc.data_ptr(), 1, 3, T, 4, out.data_ptr())
    ctx.synchronize()
    v = out.cpu().numpy()[0]
    assert np.isfinite(v).all() and v[1] < v[0] and v[1] < v[2] and v[1] < 1e-6


def test_nominal_fleet_ragged_matches_oracle(ctx):
    # several vehicles with their own physical parameters; 100 samples (not a
    # multiple of the block size)
    w = W.nominal(seed=4, batch=3, samples=100)
    domains = W.fleet_domains(4, 3)
    noise = normals(101, (1, 3, 100, 15, 4))
    r = L.MppiPlanner(ctx, w.mppi).plan(_scorer(ctx, w, domains), injected_noise=noise)
    ref = O.mppi_plan(w.mppi, 3, _oracle_fn(w, domains), noise=noise)
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"])
    assert_same_argmin(r.best_indices, ref["best"], ref["scores"])


def test_nominal_closed_loop_tracks_oracle(ctx):
    # A short closed loop (plan -> plant step -> shift warm start), GPU vs oracle.
    w = W.nominal(seed=5)
    dom = L.Domain.default()
    p = L.MppiPlanner(ctx, w.mppi)
    p.set_warm_start_sequence(w.warm_start)
    sc = L.NominalScorer(ctx, w.dt, w.trim, w.cost, w.substeps)
    x = w.initial[0].copy()
    m = w.motors[0].copy()
    warm_ref = w.warm_start.copy()
    for step in range(5):
        refs = L.reference_horizon("figure-eight", w.t0 + step * w.dt, w.dt, 15, 2.0, 8.0)[None]
        sc.set_context(x[None], m[None], refs, w.reference_actions)
        noise = normals(200 + step, (1, 1, 512, 15, 4))
        r = p.plan(sc, injected_noise=noise)
        ref = O.mppi_plan(w.mppi, 1, (O.NOMINAL_FN, O.nominal_ctx(x[None], m[None], refs, w.reference_actions,
                                                                   w.cost, w.dt, w.trim)),
                          noise=noise, warm_start=warm_ref)
        assert_actions_close(r.sequence, ref["sequence"], 2e-4)
        warm_ref = ref["warm"]
        action = ref["sequence"][0, 0]
        for _ in range(10):
            L.plant_step(dom, x, m, action, w.dt / 10)
