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


def _f(x):
    return np.float32(x)


class OracleSession:
    """The session's host logic (session.rs:241-445) over the oracle."""

    def __init__(self, cfg, initial, sky=None):
        dom = L.Domain.default()
        self.cfg, self.sky, self.dom = cfg, sky, dom
        self.hover = np.full(4, _f(dom.mass) * _f(dom.gravity) / _f(4.0), np.float32)
        self.high = _f(dom.mass) * _f(dom.gravity) * _f(dom.max_thrust_weight) / _f(4.0)
        self.H = sky.model.history_steps if sky is not None else 10
        self.mppi = L.MppiConfig(horizon=cfg.horizon, samples=cfg.samples, action_dim=4, iterations=cfg.iterations,
                                 action_bounds=L.ActionBounds.scalar(4, 0.0, float(self.high)),
                                 noise_std_per_action=list(cfg.action_noise), temperature=cfg.temperature,
                                 seed=cfg.planner_seed)
        self.reset_with_action(initial, self.hover)

    def reset_with_action(self, state, action):
        a = np.asarray(action, np.float32)
        collective = ((a[0] + a[1]) + a[2]) + a[3]
        nominal = ((self.hover[0] + self.hover[1]) + self.hover[2]) + self.hover[3]
        self.trim = collective / nominal * _f(self.cfg.trim_multiplier)
        self.motors = (a / self.trim).astype(np.float32)
        self.states = [np.asarray(state, np.float32).copy() for _ in range(self.H)]
        self.actions = [a.copy() for _ in range(self.H - 1)]
        self.active = self.pending = None
        self.offset = 0  # a fresh planner

    def commit_observation(self, state, action):
        self.active, self.pending = self.pending, None
        response = _f(1.0) - np.exp(_f(-self.cfg.dt) / _f(self.dom.motor_time_constant), dtype=np.float32)
        for i in range(4):
            target = np.clip(_f(action[i]) / self.trim, _f(0.0), self.high)
            self.motors[i] += (target - self.motors[i]) * response
        self.states = self.states[1:] + [np.asarray(state, np.float32).copy()]
        self.actions = self.actions[1:] + [np.asarray(action, np.float32).copy()]

    def plan(self, refs):
        self.pending = None
        last = self.states[-1]
        prior = np.clip(O.geometric_prior(last, refs, self.cfg.dt) * self.trim, 0.0, self.high).astype(np.float32)
        warm = prior + self.active if (self.cfg.warm_start == 1 and self.active is not None) else prior
        warm = np.clip(warm, 0.0, self.high).astype(np.float32)
        if self.sky is None:
            c = O.nominal_ctx(last[None], self.motors[None], refs[None], prior[None], self.cfg.cost, self.cfg.dt,
                              float(self.trim))
            fn = O.NOMINAL_FN
        else:
            m = O.SkyJepaModel(self.sky.model, self.sky.weights)
            self._m = m
            c = m.score_ctx((self.sky.state_mean, self.sky.state_std, self.sky.action_mean, self.sky.action_std),
                            np.stack(self.states)[None], np.stack(self.actions)[None], refs[None], prior[None],
                            self.cfg.cost, self.cfg.dt)
            fn = O.SKYJEPA_FN
        r = O.mppi_plan(self.mppi, 1, (fn, c), seed=self.cfg.planner_seed, offset=self.offset, warm_start=warm[None])
        per = self.cfg.samples * self.cfg.horizon * 4
        self.offset += (per + per % 2) * self.cfg.iterations
        if self.cfg.warm_start == 1:
            self.pending = L.shifted_residual(r["sequence"][0], prior, self.cfg.residual_limit_n)
        return r["sequence"][0], prior, float(r["scores"].min())


def _refs(t0, cfg):
    return L.reference_horizon("figure-eight", t0, cfg.dt, cfg.horizon, 2.0, 8.0)


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
    ref = OracleSession(cfg, x, sky)
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
