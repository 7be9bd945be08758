"""SkyJEPA controller-session host logic without a GPU: the reference's
shifted-residual unit test (src/models/skyjepa/session.rs:548-566) and the
paper-derived session settings (session.rs:52-64, control.rs:84-94)."""
import numpy as np
import pytest

import lewm_b200 as L


def test_shifted_residual_reference_known_answer():
    prior = np.array([[3.0], [4.0], [5.0]], np.float32)
    selected = np.array([[3.0], [7.0], [1.0]], np.float32)
    residual = L.shifted_residual(selected, prior, 2.0)
    assert residual.ravel().tolist() == [2.0, -2.0, 0.0]
    assert (np.full((3, 1), 6.0, np.float32) + residual).ravel().tolist() == [8.0, 4.0, 6.0]


def test_shifted_residual_single_step_is_zero():
    assert L.shifted_residual(np.array([[5.0, 1.0]], np.float32), np.zeros((1, 2), np.float32), 1.0).tolist() == \
        [[0.0, 0.0]]


def test_paper_session_config():
    c = L.SessionConfig.paper()
    assert (c.samples, c.horizon, c.planner_seed, c.iterations) == (512, 15, 7, 1)
    assert c.warm_start == L.WARM_STARTS["fresh_prior"] and c.dynamics == L.DYNAMICS["learned"]
    assert c.residual_limit_n == 2.0 and c.trim_multiplier == 1.0
    assert c.dt == pytest.approx(0.05) and c.temperature == pytest.approx(1e-4)
    assert list(c.action_noise) == pytest.approx([0.60, 0.15, 0.15, 0.05])
    p = L.TrackingCost.paper()
    assert (c.cost.position, c.cost.velocity, c.cost.attitude) == (p.position, p.velocity, p.attitude)
