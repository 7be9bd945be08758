"""Fused SkyJEPA learned MPPI on the GPU against the oracle
(SkyJepaMppiScorer, src/models/skyjepa/control.rs:146-317, with the
TCN/GRU/prober/integrator of model.rs, tcn.rs, prober.rs, kinematics.rs)."""
import numpy as np
import pytest

import lewm_b200 as L
import oracle as O
from gpu_helpers import assert_actions_close, assert_costs_close, assert_same_argmin, assert_same_elites, normals
from lewm_b200 import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _norm(w):
    return (w.state_mean, w.state_std, w.action_mean, w.action_std)


def _scorer(ctx, w, precision="f32"):
    sc = L.SkyJepaScorer(ctx, w.model, w.weights, w.state_mean, w.state_std, w.action_mean, w.action_std, w.cost,
                         w.dt)
    sc.set_precision(precision)
    sc.set_context(w.state_history, w.action_history, w.reference_states, w.reference_actions)
    return sc


def _oracle(w):
    m = O.SkyJepaModel(w.model, w.weights)
    c = m.score_ctx(_norm(w), w.state_history, w.action_history, w.reference_states, w.reference_actions, w.cost,
                    w.dt)
    return m, c


# "f32" takes the split-fp16 tensor-core rollout at this shape (3 launches:
# sampling + inputs, h0, rollout); "f32-cuda-core" the fused CUDA-core kernel
@pytest.mark.parametrize("precision, launches", [("f32", 3), ("f32-cuda-core", 1)])
def test_skyjepa_mppi_matches_oracle_injected_noise(ctx, precision, launches):
    w = W.skyjepa(seed=1)
    noise = normals(300, (1, 1, 512, 15, 4))
    p = L.MppiPlanner(ctx, w.mppi)
    p.set_warm_start_sequence(w.warm_start)
    sc = _scorer(ctx, w, precision)
    n0 = ctx.launch_count()
    r = p.plan(sc, injected_noise=noise)
    assert ctx.launch_count() - n0 == launches
    m, c = _oracle(w)
    ref = O.mppi_plan(w.mppi, 1, (O.SKYJEPA_FN, c), noise=noise, warm_start=w.warm_start)
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"])
    assert_same_argmin(r.best_indices, ref["best"], ref["scores"])


def test_skyjepa_predicted_states_match_oracle(ctx):
    w = W.skyjepa(seed=2, samples=64)
    cand = (w.hover + normals(6, (1, 64, 15, 4)) * 0.5).astype(np.float32)
    sc = _scorer(ctx, w)
    d = torch.as_tensor(cand).cuda()
    states = torch.empty((1, 64, 15, 18), device="cuda")
    torch.cuda.synchronize()
    sc.predict_device(d.data_ptr(), 1, 64, 15, states.data_ptr())
    ctx.synchronize()
    m, _ = _oracle(w)
    _, ref_states = m.scores(_norm(w), w.state_history, w.action_history, w.reference_states, w.reference_actions,
                             w.cost, w.dt, cand, with_states=True)
    got = states.cpu().numpy()
    assert np.abs(got - ref_states).max() < 1e-4 * max(1.0, np.abs(ref_states).max())


@pytest.mark.parametrize("latent", [256, 128])
def test_skyjepa_scores_ragged_batch(ctx, latent):
    cfg = L.SkyJepaConfig.wide()
    cfg.latent_dim = latent
    w = W.skyjepa(seed=3, batch=2, samples=100, horizon=7, config=cfg)
    cand = (w.hover + normals(7, (2, 100, 7, 4)) * 0.7).astype(np.float32)
    sc = _scorer(ctx, w)
    d = torch.as_tensor(cand).cuda()
    out = torch.empty((2, 100), device="cuda")
    torch.cuda.synchronize()
    sc.score_device(d.data_ptr(), 2, 100, 7, 4, out.data_ptr())
    ctx.synchronize()
    m, _ = _oracle(w)
    ref = m.scores(_norm(w), w.state_history, w.action_history, w.reference_states, w.reference_actions, w.cost,
                   w.dt, cand)
    assert_costs_close(out.cpu().numpy(), ref)


def test_skyjepa_cem_elites_match_oracle(ctx):
    w = W.skyjepa(seed=4, samples=128)
    cfg = L.CemConfig(horizon=15, samples=128, elites=16, action_dim=4, iterations=2,
                      action_bounds=L.ActionBounds.scalar(4, 0.0, 2 * w.hover), init_std=0.5, seed=3)
    noise = normals(400, (2, 1, 128, 15, 4))
    planner = L.CemPlanner(ctx, cfg)
    r = planner.plan(_scorer(ctx, w), injected_noise=noise)
    m, c = _oracle(w)
    ref = O.cem_plan(cfg, 1, (O.SKYJEPA_FN, c), noise=noise)
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"], 1e-4)
    # the elite index set of every iteration (select_elites, src/planner.rs:1730-1754)
    assert assert_same_elites(planner.elite_indices(), ref["elites"], ref["iteration_scores"]) == 2
