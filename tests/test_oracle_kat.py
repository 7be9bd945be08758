"""The CPU oracle against the reference's own known-answer tests.

Each test restates one reference test (path:line in le-wm-nv) on the oracle,
with the reference's inputs and expected values.  The reference cannot run in
this image (Rust, no toolchain), so these are what pins the oracle.
"""
import numpy as np
import pytest

import oracle as O
from lewm_b200 import (CemConfig, Domain, IcemConfig, KinematicConfig, MppiConfig, SkyJepaConfig, TcnConfig,
                       TrackingCost, hover_state)


# ---------------------------------------------------------------- planner

def test_lowest_score_indices_returns_requested_count():
    # src/planner.rs:1922-1930
    scores = np.array([[3, 1, 4, 0.5], [9, -1, 2, -2]], np.float32)
    assert O.lowest_k(scores, 3).tolist() == [[3, 1, 0], [3, 1, 2]]


def test_lowest_score_indices_covers_benchmark_sample_count():
    # src/planner.rs:1932-1941
    scores = np.array([[1024 - i for i in range(1024)]], np.float32)
    assert O.lowest_k(scores, 4).tolist() == [[1023, 1022, 1021, 1020]]


def test_lowest_k_nan_ranks_last_and_ties_take_lower_index():
    # swm_lowest_k_indices_f32 semantics (src/planner.rs:1811, 1830-1833)
    scores = np.array([[np.nan, 2.0, 1.0, 1.0, -0.0, 0.0, np.inf]], np.float32)
    # NaN becomes +inf and ties with the real +inf: the lower index (0) ranks first
    assert O.lowest_k(scores, 7).tolist() == [[4, 5, 2, 3, 1, 0, 6]]


def test_select_elites_gathers_per_batch():
    # src/planner.rs:1902-1920
    cand = np.arange(8, dtype=np.float32).reshape(2, 4, 1, 1)
    scores = np.array([[3, 1, 4, 0.5], [9, -1, 2, -2]], np.float32)
    idx = O.lowest_k(scores, 2)
    assert O.gather(cand, idx).reshape(2, 2).tolist() == [[3, 1], [7, 5]]
    best = O.lowest_k(scores, 1)
    assert best[:, 0].tolist() == [3, 3]
    assert O.gather(cand, best).reshape(2).tolist() == [3, 7]


def test_temporal_colored_noise_is_finite_and_standardised():
    # src/planner.rs:1943-1953 (finite); the kernel standardises every lane.
    noise = O.normals(11, 0, 2 * 8 * 6 * 4).reshape(2, 8, 6, 4)
    col = O.color_noise(noise, 2.0)
    assert col.shape == (2, 8, 6, 4) and np.isfinite(col).all()
    lanes = col.transpose(0, 1, 3, 2).reshape(-1, 6)
    assert np.abs(lanes.mean(axis=1)).max() < 1e-5
    assert np.abs((lanes ** 2).mean(axis=1) - 1.0).max() < 1e-4
    assert np.array_equal(O.color_noise(noise, 0.0), noise)


def test_sampled_candidates_include_mean_in_first_slot():
    # src/planner.rs:1955-1979
    mean = np.array([[[0.25, -0.5], [0.75, 0.1]]], np.float32)
    std = np.full((1, 2, 2), 0.5, np.float32)
    noise = O.normals(5, 0, 4 * 2 * 2).reshape(1, 4, 2, 2)
    cand = O.sample(mean, std, noise, [-1, -1], [1, 1])
    assert np.array_equal(cand[0, 0], mean[0])
    assert (cand >= -1).all() and (cand <= 1).all()


def test_carried_elites_replace_samples_without_growing_candidate_count():
    # src/planner.rs:1981-1995
    cand = np.arange(5, dtype=np.float32).reshape(1, 5, 1, 1)
    carried = np.array([[[[10.0]], [[11.0]]]], np.float32)
    out = O.inject_carried(cand, carried, 2)
    assert out.shape == (1, 5, 1, 1)
    assert out.reshape(5).tolist() == [0, 10, 11, 3, 4]


def _fixed_scores(cand):
    # FixedScoreScorer (src/planner.rs:2000-2020): score = index, slot 0 = 100
    B, S = cand.shape[:2]
    s = np.tile(np.arange(S, dtype=np.float32), (B, 1))
    s[:, 0] = 100.0
    return s


def test_icem_returns_final_mean_sequence_not_best_sample():
    # src/planner.rs:1997-2043
    cfg = IcemConfig(horizon=2, samples=4, elites=2, action_dim=1, iterations=1, keep_elites=0, alpha=1.0,
                     init_std=0.5, seed=123)
    warm = np.array([[[0.25], [-0.5]]], np.float32)
    r = O.icem_plan(cfg, 1, _fixed_scores, seed=123, warm_start=warm)
    assert r["best"].tolist() == [1]
    assert np.array_equal(r["sequence"], warm)


def test_icem_can_return_best_sample_sequence():
    # src/planner.rs:2045-2092
    cfg = IcemConfig(horizon=2, samples=4, elites=2, action_dim=1, iterations=1, keep_elites=0, alpha=1.0,
                     init_std=0.5, seed=123, return_mean=False)
    warm = np.array([[[0.25], [-0.5]]], np.float32)
    r = O.icem_plan(cfg, 1, _fixed_scores, seed=123, warm_start=warm)
    assert r["best"].tolist() == [1]
    assert not np.array_equal(r["sequence"], warm)
    assert np.array_equal(r["sequence"][0], r["candidates"][0, 1])


def test_mppi_uses_per_action_noise_and_shifts_warm_start():
    # src/planner.rs:2094-2137 (SumScorer, one sample: the mean comes back exactly)
    cfg = MppiConfig(horizon=3, samples=1, action_dim=2, noise_std_per_action=[0.6, 0.1], seed=9)
    initial = np.array([[[0.1, 0.2], [0.3, 0.4], [0.5, 0.6]]], np.float32)
    r = O.mppi_plan(cfg, 1, lambda c: (c ** 2).sum(axis=(2, 3)), seed=9, warm_start=initial)
    assert np.array_equal(r["sequence"], initial)
    assert np.array_equal(r["warm"], np.array([[[0.3, 0.4], [0.5, 0.6], [0.5, 0.6]]], np.float32))


def test_cem_refit_is_unbiased_and_floored():
    # elites.mean(1), elites.var(1) (unbiased), enforce_min_std (src/planner.rs:516-517, 1618-1626)
    el = np.array([[[[1.0]], [[3.0]]]], np.float32)
    mean, std = O.refit(el, 0.0)
    assert mean.item() == 2.0 and abs(std.item() - np.sqrt(2.0)) < 1e-6
    same = np.array([[[[1.0]], [[1.0]]]], np.float32)
    mean, std = O.refit(same, 1e-3)
    assert std.item() == np.float32(1e-3)


def test_cem_plan_converges_on_quadratic():
    cfg = CemConfig(horizon=4, samples=64, elites=8, action_dim=2, iterations=6, seed=3)
    target = np.array([0.3, -0.2], np.float32)
    r = O.cem_plan(cfg, 1, lambda c: ((c - target) ** 2).sum(axis=(2, 3)), seed=3)
    assert np.abs(r["sequence"] - target).max() < 0.1


def test_philox_normals_are_standard_normal():
    z = O.normals(2024, 7, 1 << 18)
    assert abs(z.mean()) < 0.01 and abs(z.std() - 1.0) < 0.01
    assert np.array_equal(O.normals(2024, 7 + 5, 10), z[5:15])


# ---------------------------------------------------------------- rotor physics

def test_sampled_domains_stay_in_reported_ranges():
    # tests/skyjepa_sim.rs:3-18
    nominal = Domain.default()
    for seed in range(100):
        d = Domain.sample(seed)
        assert nominal.mass * 0.5 <= d.mass <= nominal.mass * 1.5
        assert 0.01 <= d.motor_time_constant <= 0.1
        assert all(0.1 <= v <= 0.5 for v in d.drag)
        assert 0.5 <= d.thrust_scale <= 1.5 and 0.5 <= d.torque_scale <= 1.5


def test_nominal_rotor_plant_hovers():
    # tests/skyjepa_sim.rs:20-34
    d = Domain.default()
    x = hover_state()
    m = np.full(4, d.hover_force(), np.float32)
    for _ in range(1000):
        O.plant_step(d, x, m, np.full(4, d.hover_force(), np.float32), 0.001)
    assert abs(x[2] - 1.0) < 1e-3
    assert np.abs(x[3:6]).max() < 1e-3 and np.abs(x[15:18]).max() < 1e-3


@pytest.mark.parametrize("domain_seed", [None, 918])
def test_fused_nominal_candidates_match_the_cpu_rigid_body_plant(domain_seed):
    # tests/skyjepa_nominal.rs:8-51: CUDA-branch restatement vs CPU plant < 2e-3
    d = Domain.default() if domain_seed is None else Domain.sample(domain_seed)
    s = hover_state()
    s[3:6] = [0.3, -0.2, 0.1]
    s[15:18] = [0.05, -0.02, 0.03]
    batch, horizon = 5, 30
    hover = d.hover_force()
    initial = np.tile(s, (batch, 1))
    motors = np.full((batch, 4), hover, np.float32)
    i = np.arange(batch * horizon * 4, dtype=np.float32)
    actions = (hover + 0.02 * np.sin(i * np.float32(0.71))).astype(np.float32).reshape(batch, horizon, 4)
    plant = O.nominal_rollout(initial, actions, motors, 0.05, 10, d)
    kernel = O.nominal_rollout(initial, actions, motors, 0.05, 10, d, kernel_form=True)
    assert np.abs(plant - kernel).max() < 2e-3


@pytest.mark.parametrize("trim", [1.0, 2.0])
def test_nominal_scorer_uses_observed_trim_and_the_shared_tracking_cost(trim):
    # tests/skyjepa_nominal.rs:84-115
    d = Domain.default()
    hover = d.mass * d.gravity / 4.0
    s = hover_state()
    horizon = 15
    cand = np.concatenate([np.full((1, 1, horizon, 4), hover * trim + delta, np.float32)
                           for delta in (0.5, 0.0, -0.5)], axis=1)
    scores = O.nominal_scores(s[None], np.full((1, 4), hover, np.float32), np.tile(s, (1, horizon, 1)),
                              np.full((1, horizon, 4), hover * trim, np.float32), TrackingCost.paper(), 0.05, trim,
                              cand)
    assert np.isfinite(scores).all()
    assert scores[0, 1] < scores[0, 0] and scores[0, 1] < scores[0, 2]
    assert scores[0, 1] < 1e-6


# ---------------------------------------------------------------- integrator

def test_so3_exponential_preserves_rotation_geometry():
    # tests/skyjepa.rs:110-125
    for w in ([0.0, 0.0, 0.0], [0.2, -0.1, 0.3]):
        R = O.so3_exp(w)
        assert np.abs(np.linalg.norm(R, axis=1) - 1.0).max() < 1e-4
        assert abs(float(R[0] @ R[1])) < 1e-4


def _rotor_kin():
    return KinematicConfig(1.3, 9.81, 0.2, 1)


def test_nominal_rotor_hover_remains_stationary():
    # tests/skyjepa.rs:127-164 (both integrator restatements)
    s = hover_state()[None]
    f = np.float32(1.3) * np.float32(9.81) / np.float32(4.0)
    actions = np.full((1, 3, 4), f, np.float32)
    dt = np.full((1, 3), 0.05, np.float32)
    for ref in (False, True):
        out = O.integrate(s, actions, dt, np.zeros((1, 3, 3), np.float32), np.zeros((1, 3, 12), np.float32),
                          _rotor_kin(), reference_form=ref)
        assert np.abs(out[0, :, 2] - 1.0).max() < 1e-5
        assert np.abs(out[0, :, 3:6]).max() < 1e-5


def test_fused_integrator_matches_training_integrator():
    # tests/skyjepa.rs:166-207: fused-kernel restatement vs differentiable integrator < 2e-5
    rng = np.random.default_rng(0)
    batch, steps = 5, 4
    init = np.zeros((batch, 18), np.float32)
    init[:, 0] = 0.3; init[:, 2] = 1.2; init[:, 3] = 0.1; init[:, 5] = -0.05
    init[:, 6] = init[:, 10] = init[:, 14] = 1.0
    init[:, 15] = 0.02; init[:, 16] = -0.03; init[:, 17] = 0.01
    actions = rng.uniform(2.5, 3.8, (batch, steps, 4)).astype(np.float32)
    dt = np.full((batch, steps), 0.05, np.float32)
    res = rng.normal(0, 0.1, (batch, steps, 3)).astype(np.float32)
    maps = rng.normal(0, 0.02, (batch, steps, 12)).astype(np.float32)
    a = O.integrate(init, actions, dt, res, maps, _rotor_kin())
    b = O.integrate(init, actions, dt, res, maps, _rotor_kin(), reference_form=True)
    assert np.abs(a - b).max() < 2e-5


# ---------------------------------------------------------------- model

def _tiny_config():
    # tests/skyjepa.rs:15-32
    c = SkyJepaConfig()
    c.state_dim, c.action_dim, c.history_steps, c.rollout_steps, c.latent_dim = 6, 2, 4, 3, 6
    c.state_encoder = TcnConfig(6, 2, (4, 6, 0, 0, 0, 0, 0, 0), 3)
    c.action_encoder = TcnConfig(2, 2, (3, 4, 0, 0, 0, 0, 0, 0), 3)
    c.prober_hidden_dim, c.prober_hidden_layers = 32, 2
    c.kinematics = _rotor_kin()
    return c


def test_paper_configuration_matches_reported_dimensions():
    # tests/skyjepa.rs:34-45
    c = SkyJepaConfig.paper()
    assert (c.state_dim, c.action_dim, c.history_steps, c.rollout_steps, c.latent_dim) == (18, 4, 10, 20, 24)
    assert list(c.state_encoder.channels[:3]) == [8, 8, 16]
    assert list(c.action_encoder.channels[:3]) == [4, 4, 8]


def test_candidate_rollout_batches_samples_and_windows():
    # tests/skyjepa.rs:79-108 (shapes, finiteness) on the tiny config
    cfg = _tiny_config()
    rng = np.random.default_rng(1)
    w = rng.normal(0, 0.3, O.skyjepa_weight_count(cfg)).astype(np.float32)
    m = O.SkyJepaModel(cfg, w)
    states = rng.normal(size=(2, 4, 6)).astype(np.float32)
    ah = rng.normal(size=(2, 3, 2)).astype(np.float32)
    cand = rng.normal(size=(2, 5, 3, 2)).astype(np.float32)
    lat = m.rollout_latents(states, ah, cand)
    assert lat.shape == (2, 5, 3, 6) and np.isfinite(lat).all()


def test_tcn_windows_are_padded_independently():
    # model.rs:192-204 / tcn.rs:36-43: a window's output depends only on its own
    # 10 steps (left zero padding per window), so a window equals a fresh call.
    cfg = SkyJepaConfig.paper()
    rng = np.random.default_rng(2)
    m = O.SkyJepaModel(cfg, rng.normal(0, 0.2, O.skyjepa_weight_count(cfg)).astype(np.float32))
    hist = rng.normal(size=(1, 9, 4)).astype(np.float32)
    cand = rng.normal(size=(1, 1, 3, 4)).astype(np.float32)
    seq = np.concatenate([hist[0], cand[0, 0]], axis=0)
    windows = np.stack([seq[t:t + 10] for t in range(3)])
    emb = m.tcn_last(1, windows)
    emb0 = m.tcn_last(1, windows[:1])
    assert np.array_equal(emb[0], emb0[0])


def test_gru_step_matches_pytorch_gate_convention():
    # candle_nn GRU::step: gate order r, z, n; h' = z*h - (z-1)*n
    import torch
    cfg = SkyJepaConfig.paper()
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.3, O.skyjepa_weight_count(cfg)).astype(np.float32)
    m = O.SkyJepaModel(cfg, w)
    H, E = 24, 8
    # locate the GRU tensors in the blob (layout of include/lewm_b200.h)
    n_state = 0
    ins = 18
    for ch in (8, 8, 16):
        n_state += ch * ins * 3 + ch + ch * ch * 3 + ch + (ch * ins + ch if ins != ch else 0)
        ins = ch
    off = n_state + H * 16 + H
    ins = 4
    for ch in (4, 4, 8):
        off += ch * ins * 3 + ch + ch * ch * 3 + ch + (ch * ins + ch if ins != ch else 0)
        ins = ch
    w_ih = w[off:off + 3 * H * E].reshape(3 * H, E); off += 3 * H * E
    w_hh = w[off:off + 3 * H * H].reshape(3 * H, H); off += 3 * H * H
    b_ih = w[off:off + 3 * H]; off += 3 * H
    b_hh = w[off:off + 3 * H]
    gru = torch.nn.GRUCell(E, H)
    with torch.no_grad():
        gru.weight_ih.copy_(torch.from_numpy(w_ih)); gru.weight_hh.copy_(torch.from_numpy(w_hh))
        gru.bias_ih.copy_(torch.from_numpy(b_ih)); gru.bias_hh.copy_(torch.from_numpy(b_hh))
    x = rng.normal(size=(3, E)).astype(np.float32)
    h = rng.normal(size=(3, H)).astype(np.float32)
    ours = m.gru_step(x, h)
    with torch.no_grad():
        ref = gru(torch.from_numpy(x), torch.from_numpy(h)).numpy()
    assert np.abs(ours - ref).max() < 1e-5

    # the tensor-core rounding model: the same cell fed bf16 weights, bf16
    # x and a bf16 copy of h (f32 h in the update), one bf16 bias per r / z row
    def bf(a):
        return torch.from_numpy(np.asarray(a, np.float32)).to(torch.bfloat16).to(torch.float32)

    mq = O.SkyJepaModel(cfg, w, tensor_core_rounding=True)
    ours_q = mq.gru_step(x, h)
    wi, wh = bf(w_ih), bf(w_hh)
    xq, hq, hf = bf(x), bf(h), torch.from_numpy(h)
    b_rz = bf(b_ih[:2 * H] + b_hh[:2 * H])
    gi = xq @ wi.T
    gh = hq @ wh.T
    r = torch.sigmoid(gi[:, :H] + gh[:, :H] + b_rz[:H])
    z = torch.sigmoid(gi[:, H:2 * H] + gh[:, H:2 * H] + b_rz[H:])
    n = torch.tanh(gi[:, 2 * H:] + bf(b_ih[2 * H:]) + r * (gh[:, 2 * H:] + bf(b_hh[2 * H:])))
    ref_q = (z * hf - (z - 1.0) * n).numpy()
    assert np.abs(ours_q - ref_q).max() < 1e-5
    assert np.abs(ours_q - ours).max() > 1e-4   # the rounding is actually applied


# ---------------------------------------------------------------- task

def test_geometric_hover_prior_balances_nominal_rotors():
    # src/skyjepa_task.rs:298-310
    s = O.reference_state(0, 0.0, 2.0, 8.0)
    actions = O.geometric_prior(s, np.tile(s, (15, 1)), 0.05)
    assert np.abs(actions - 1.3 * 9.81 / 4.0).max() < 1e-5


def test_reference_trajectories():
    # src/skyjepa_task.rs:276-296
    circle = O.reference_state(1, 0.0, 2.0, 8.0)
    assert circle[0:3].tolist() == [0.0, 0.0, 1.0]
    assert circle[8] < 0.0 and circle[14] < 1.0


def test_icem_trace_records_the_reference_scores():
    # IcemPlanner::trace_device (src/planner.rs:900-1010): the plan itself is
    # the plain iCEM plan; per iteration it records the mean's score, the best
    # candidate score, the elite mean's score and the updated mean's score.
    cfg = IcemConfig(horizon=5, samples=48, elites=6, action_dim=2, keep_elites=2, iterations=3, noise_beta=1.0,
                     alpha=0.2, seed=9)
    target = np.array([0.3, -0.4], np.float32)

    def quad(c):
        return ((c - target) ** 2).sum(axis=(2, 3))

    warm = np.full((2, 5, 2), 0.05, np.float32)
    plan = O.icem_plan(cfg, 2, quad, seed=9, warm_start=warm)
    tr = O.icem_trace(cfg, 2, quad, seed=9, warm_start=warm)
    assert np.array_equal(tr["sequence"], plan["sequence"])
    assert np.array_equal(tr["scores"], plan["scores"])
    assert tr["trace"].shape == (3, 4, 2)
    assert np.allclose(tr["trace"][0, 0], quad(warm[:, None])[:, 0], rtol=1e-6)
    assert np.array_equal(tr["trace"][-1, 1], tr["scores"].min(axis=1))
    # the final mean (return_mean) is the last updated mean
    assert np.allclose(tr["trace"][-1, 3], quad(tr["sequence"][:, None])[:, 0], rtol=1e-6)
