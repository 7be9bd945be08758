"""The small-latent SkyJEPA path (latent <= 64: the paper-derived model of
src/models/skyjepa/config.rs:59-77, latent 24, TCN [8, 8, 16] / [4, 4, 8],
prober 32 x 2) on the GPU against the oracle: scores, predicted states,
MPPI and CEM plans, shapes that use both register halves of a lane."""
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


def _scorer(ctx, w, masses=None):
    sc = L.SkyJepaScorer(ctx, w.model, w.weights, w.state_mean, w.state_std, w.action_mean, w.action_std, w.cost,
                         w.dt)
    sc.set_context(w.state_history, w.action_history, w.reference_states, w.reference_actions, vehicle_mass=masses)
    return sc


def _oracle(w, masses=None):
    m = O.SkyJepaModel(w.model, w.weights)
    c = m.score_ctx(_norm(w), w.state_history, w.action_history, w.reference_states, w.reference_actions, w.cost,
                    w.dt, masses=masses)
    return m, c


def _variant(latent, hid, layers, hist, kernel, state_ch, action_ch):
    c = L.SkyJepaConfig.paper()
    c.latent_dim, c.prober_hidden_dim, c.prober_hidden_layers, c.history_steps = latent, hid, layers, hist
    c.state_encoder.kernel_size = c.action_encoder.kernel_size = kernel
    c.state_encoder.levels, c.action_encoder.levels = len(state_ch), len(action_ch)
    for i, v in enumerate(state_ch):
        c.state_encoder.channels[i] = v
    for i, v in enumerate(action_ch):
        c.action_encoder.channels[i] = v
    return c


def _scores(ctx, sc, cand):
    B, S, T, A = cand.shape
    d = torch.as_tensor(cand).cuda()
    out = torch.empty((B, S), device="cuda")
    torch.cuda.synchronize()
    sc.score_device(d.data_ptr(), B, S, T, A, out.data_ptr())
    ctx.synchronize()
    return out.cpu().numpy()


CONFIGS = {
    "paper": L.SkyJepaConfig.paper,
    "latent48-hid40-3layers": lambda: _variant(48, 40, 3, 6, 2, [8, 12], [4, 6]),
    "latent64-hid64-1layer": lambda: _variant(64, 64, 1, 12, 3, [16, 16, 32, 32], [4, 8, 8, 8]),
    "latent8-hid12": lambda: _variant(8, 12, 2, 3, 3, [4], [4]),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_small_scores_match_oracle(ctx, name):
    w = W.skyjepa(seed=11, batch=2, samples=37, horizon=9, config=CONFIGS[name]())
    cand = (w.hover + normals(81, (2, 37, 9, 4)) * 0.6).astype(np.float32)
    got = _scores(ctx, _scorer(ctx, w), cand)
    m, _ = _oracle(w)
    ref = m.scores(_norm(w), w.state_history, w.action_history, w.reference_states, w.reference_actions, w.cost,
                   w.dt, cand)
    assert_costs_close(got, ref)


def test_small_predicted_states_and_masses(ctx):
    w = W.skyjepa(seed=12, batch=3, samples=20, horizon=15, config=L.SkyJepaConfig.paper())
    masses = np.array([1.1, 1.3, 1.55], np.float32)
    cand = (w.hover + normals(82, (3, 20, 15, 4)) * 0.5).astype(np.float32)
    sc = _scorer(ctx, w, masses)
    d = torch.as_tensor(cand).cuda()
    states = torch.empty((3, 20, 15, 18), device="cuda")
    torch.cuda.synchronize()
    sc.predict_device(d.data_ptr(), 3, 20, 15, states.data_ptr())
    ctx.synchronize()
    m, _ = _oracle(w)
    ref_scores, ref_states = m.scores(_norm(w), w.state_history, w.action_history, w.reference_states,
                                      w.reference_actions, w.cost, w.dt, cand, with_states=True, masses=masses)
    got = states.cpu().numpy()
    assert np.abs(got - ref_states).max() < 1e-4 * max(1.0, np.abs(ref_states).max())
    assert_costs_close(_scores(ctx, sc, cand), ref_scores)


def test_small_mppi_matches_oracle(ctx):
    # the reference's published workload: paper model, 512 x 15, one MPPI iteration
    w = W.skyjepa(seed=13, config=L.SkyJepaConfig.paper())
    noise = normals(83, (1, 1, 512, 15, 4))
    p = L.MppiPlanner(ctx, w.mppi)
    p.set_warm_start_sequence(w.warm_start)
    n0 = ctx.launch_count()
    r = p.plan(_scorer(ctx, w), injected_noise=noise)
    assert ctx.launch_count() - n0 == 4  # sample, inputs, h0, rollout (MPPI fused)
    m, c = _oracle(w)
    ref = O.mppi_plan(w.mppi, 1, (O.SKYJEPA_FN, c), noise=noise, warm_start=w.warm_start)
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"])
    assert_same_argmin(r.best_indices, ref["best"], ref["scores"])


def test_small_seeded_mppi_matches_oracle(ctx):
    w = W.skyjepa(seed=14, batch=2, samples=300, horizon=12, config=L.SkyJepaConfig.paper())
    p = L.MppiPlanner(ctx, w.mppi)
    p.set_warm_start_sequence(w.warm_start)
    r = p.plan(_scorer(ctx, w))
    m, c = _oracle(w)
    ref = O.mppi_plan(w.mppi, 2, (O.SKYJEPA_FN, c), seed=w.mppi.seed, warm_start=w.warm_start)
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"])


def test_small_cem_matches_oracle(ctx):
    w = W.skyjepa(seed=15, samples=128, config=L.SkyJepaConfig.paper())
    cfg = L.CemConfig(horizon=15, samples=128, elites=16, action_dim=4, iterations=2,
                      action_bounds=L.ActionBounds.scalar(4, 0.0, 2 * w.hover), init_std=0.5, seed=3)
    noise = normals(84, (2, 1, 128, 15, 4))
    r = L.CemPlanner(ctx, cfg).plan(_scorer(ctx, w), injected_noise=noise)
    m, c = _oracle(w)
    ref = O.cem_plan(cfg, 1, (O.SKYJEPA_FN, c), noise=noise)
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"], 1e-4)
