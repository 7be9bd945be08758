"""SkyJepaControllerSession (src/models/skyjepa/session.rs:110-470) on the
GPU against the same session restated here over the oracle's planner,
scorers and geometric prior, in closed loop with the host rotor plant.

The paper temperature (1e-4) makes MPPI pick essentially one candidate, so a
near-tie in cost (well inside the 1e-4 relative cost tolerance) would swap
the chosen sequence; the closed-loop comparisons run at temperature 1."""
import numpy as np
import pytest

import lewm_b200 as L
import oracle as O
from gpu_helpers import assert_actions_close
from lewm_b200 import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _refs(t0, cfg):
    return O.reference_horizon(2, t0, cfg.dt, cfg.horizon, 2.0, 8.0)


def _closed_loop(ctx, cfg, steps, sky=None):
    dom = L.Domain.default()
    rng = np.random.default_rng(5)
    x = L.hover_state()
    x[:3] += rng.uniform(-0.2, 0.2, 3).astype(np.float32)
    if sky is None:
        sess = L.SkyJepaSession(ctx, cfg, x)
    else:
        sess = L.SkyJepaSession(ctx, cfg, x, sky.model, sky.weights, sky.state_mean, sky.state_std,
                                sky.action_mean, sky.action_std)
    ref = O.SkyJepaSession(cfg, x, None if sky is None else
                           (sky.model, sky.weights, (sky.state_mean, sky.state_std, sky.action_mean, sky.action_std)))
    motors = np.full(4, dom.mass * dom.gravity / 4, np.float32)
    for k in range(steps):
        refs = _refs(0.05 * k, cfg)
        got = sess.plan(refs)
        seq, prior, best = ref.plan(refs)
        np.testing.assert_allclose(got.prior_action, prior[0], rtol=1e-6, atol=1e-6)
        assert_actions_close(got.action_sequence, seq)
        assert got.best_candidate_score == pytest.approx(best, rel=1e-4)
        assert np.allclose(got.action_correction, got.action - got.prior_action)
        # the vehicle flies the GPU session's action; both sessions see that state
        for _ in range(10):
            L.plant_step(dom, x, motors, got.action, cfg.dt / 10)
        sess.commit_observation(x, got.action)
        ref.commit_observation(x, got.action)
    return sess


@pytest.mark.parametrize("warm", ["fresh_prior", "shifted_residual"])
def test_nominal_session_closed_loop_matches_oracle(ctx, warm):
    cfg = L.SessionConfig.paper()
    cfg.dynamics = L.DYNAMICS["nominal_physics"]
    cfg.warm_start = L.WARM_STARTS[warm]
    cfg.temperature = 1.0
    _closed_loop(ctx, cfg, 4).close()


def test_learned_session_closed_loop_matches_oracle(ctx):
    sky = W.skyjepa(seed=41)
    cfg = L.SessionConfig.paper()
    cfg.temperature = 1.0
    cfg.warm_start = L.WARM_STARTS["shifted_residual"]
    _closed_loop(ctx, cfg, 3, sky).close()


def test_prediction_and_trim(ctx):
    cfg = L.SessionConfig.paper()
    cfg.dynamics = L.DYNAMICS["nominal_physics"]
    cfg.temperature = 1.0
    x = L.hover_state()
    sess = L.SkyJepaSession(ctx, cfg, x)
    dom = L.Domain.default()
    hover = dom.mass * dom.gravity / 4
    held = np.array([1.1, 1.0, 0.9, 1.2], np.float32) * hover
    sess.reset_with_action(x, held)
    assert sess.trim_scale == pytest.approx(float(held.sum() / (4 * hover)), rel=1e-6)
    refs = _refs(0.0, cfg)
    got = sess.plan(refs, include_prediction=True)
    motors = (held / np.float32(sess.trim_scale)).astype(np.float32)
    prior = np.clip(O.geometric_prior(x, refs, cfg.dt) * np.float32(sess.trim_scale), 0.0,
                    dom.mass * dom.gravity * dom.max_thrust_weight / 4).astype(np.float32)
    _, states = O.nominal_scores(x[None], motors[None], refs[None], prior[None], cfg.cost, cfg.dt, sess.trim_scale,
                                 got.action_sequence[None, None], with_states=True)
    np.testing.assert_allclose(got.predicted_states, states[0, 0], rtol=1e-4, atol=1e-4)
    sess.close()


def test_session_validation(ctx):
    cfg = L.SessionConfig.paper()
    cfg.dynamics = L.DYNAMICS["nominal_physics"]
    x = L.hover_state()
    bad = L.SessionConfig.paper()
    bad.residual_limit_n = 0.0
    with pytest.raises(L.LwmError, match="warm-start residual limit must be finite and positive"):
        L.SkyJepaSession(ctx, bad, x)
    with pytest.raises(L.LwmError, match="learned dynamics need the model"):
        L.SkyJepaSession(ctx, L.SessionConfig.paper(), x)
    sess = L.SkyJepaSession(ctx, cfg, x)
    with pytest.raises(L.LwmError, match="SkyJEPA initial action must be finite and non-negative"):
        sess.reset_with_action(x, [1.0, -1.0, 1.0, 1.0])
    with pytest.raises(L.LwmError, match="initial trim must have positive collective force"):
        sess.reset_with_action(x, [0.0, 0.0, 0.0, 0.0])
    sess.close()
