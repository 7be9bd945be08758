"""The fleet control loop on the device: the plant of every vehicle
(SkyJepaRotorPlant::step, src/skyjepa_sim.rs:206-281), the per-step context
(commit_observation's history shift, skyjepa_reference_horizon, the geometric
prior; src/models/skyjepa/session.rs:301-400, src/skyjepa_task.rs:44-240)
and a closed loop of plan -> plant -> context, against the oracle."""
import numpy as np
import pytest

import lewm_b200 as L
import oracle as O
from gpu_helpers import assert_actions_close
from lewm_b200 import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _dev(a):
    return torch.as_tensor(np.ascontiguousarray(a)).cuda()


def _domains(B, seed):
    doms = [L.Domain.sample(seed + 31 * b) for b in range(B)]
    raw = np.frombuffer(b"".join(bytes(d) for d in doms), dtype=np.float32).reshape(B, -1)
    return doms, _dev(raw)


def test_plant_matches_oracle(ctx):
    B = 64
    doms, d_dom = _domains(B, 5)
    rng = np.random.default_rng(1)
    x = np.stack([L.hover_state() for _ in range(B)])
    x[:, :3] += rng.uniform(-0.2, 0.2, (B, 3)).astype(np.float32)
    motors = np.stack([np.full(4, d.mass * d.gravity / 4, np.float32) for d in doms])
    dx, dm = _dev(x), _dev(motors)
    ref_x, ref_m = x.copy(), motors.copy()
    for k in range(20):
        cmd = (motors * (1.0 + 0.3 * rng.standard_normal((B, 4)))).astype(np.float32)
        dc = _dev(cmd)
        torch.cuda.synchronize()
        L.plant_step_device(ctx, d_dom.data_ptr(), dx.data_ptr(), dm.data_ptr(), dc.data_ptr(), 4, B, 0.005, 10)
        ctx.synchronize()
        for b in range(B):
            for _ in range(10):
                O.plant_step(doms[b], ref_x[b], ref_m[b], cmd[b], 0.005)
    np.testing.assert_allclose(dx.cpu().numpy(), ref_x, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(dm.cpu().numpy(), ref_m, rtol=1e-5, atol=1e-5)


def _step(B, T, H, time, kind, trim, state, last_action, sh, ah, rs, ra):
    s = L.FleetStep()
    s.batch, s.horizon, s.history, s.time, s.dt = B, T, H, time, 0.05
    s.reference_kind, s.radius, s.period = kind, 2.0, 8.0
    s.prior_domain = L.Domain.default()
    s.trim = trim.data_ptr() if trim is not None else None
    s.state = state.data_ptr()
    s.last_action = last_action.data_ptr() if last_action is not None else None
    s.last_action_stride = 4
    s.state_history, s.action_history = sh.data_ptr(), ah.data_ptr()
    s.reference_states, s.reference_actions = rs.data_ptr(), ra.data_ptr()
    return s


@pytest.mark.parametrize("kind", [0, 1, 2])
def test_control_step_matches_host_session_logic(ctx, kind):
    B, T, H = 5, 15, 10
    rng = np.random.default_rng(kind)
    sh = rng.standard_normal((B, H, 18)).astype(np.float32)
    ah = rng.standard_normal((B, H - 1, 4)).astype(np.float32)
    state = np.stack([L.hover_state() for _ in range(B)])
    state[:, :6] += rng.uniform(-0.3, 0.3, (B, 6)).astype(np.float32)
    act = rng.uniform(2.0, 4.0, (B, 4)).astype(np.float32)
    trim = rng.uniform(0.9, 1.2, B).astype(np.float32)
    d_sh, d_ah, d_state, d_act, d_trim = _dev(sh), _dev(ah), _dev(state), _dev(act), _dev(trim)
    d_rs = torch.empty((B, T, 18), device="cuda")
    d_ra = torch.empty((B, T, 4), device="cuda")
    torch.cuda.synchronize()
    L.fleet_control_step_device(ctx, _step(B, T, H, 1.35, kind, d_trim, d_state, d_act, d_sh, d_ah, d_rs, d_ra))
    ctx.synchronize()
    # commit_observation shifts; the references and the trim-scaled prior follow
    np.testing.assert_array_equal(d_sh.cpu().numpy(), np.concatenate([sh[:, 1:], state[:, None]], 1))
    np.testing.assert_array_equal(d_ah.cpu().numpy(), np.concatenate([ah[:, 1:], act[:, None]], 1))
    dom = L.Domain.default()
    high = np.float32(dom.mass) * np.float32(dom.gravity) * np.float32(dom.max_thrust_weight) / np.float32(4.0)
    for b in range(B):
        refs = O.reference_horizon(kind, 1.35, 0.05, T, 2.0, 8.0)
        np.testing.assert_allclose(d_rs.cpu().numpy()[b], refs, rtol=1e-5, atol=2e-6)
        prior = np.clip(O.geometric_prior(state[b], refs, 0.05) * trim[b], 0.0, high)
        np.testing.assert_allclose(d_ra.cpu().numpy()[b], prior, rtol=1e-4, atol=1e-4)
    # the first step has no executed action yet: the histories stay
    d_sh2 = _dev(sh)
    L.fleet_control_step_device(ctx, _step(B, T, H, 0.0, kind, None, d_state, None, d_sh2, d_ah, d_rs, d_ra))
    ctx.synchronize()
    np.testing.assert_array_equal(d_sh2.cpu().numpy(), sh)


def test_fleet_closed_loop_matches_oracle(ctx):
    # paper model (small-latent path), 4 vehicles with their own domains, 5
    # control steps: context -> warm start -> plan -> plant, all on the device
    B, S, T, steps = 4, 256, 15, 5
    w = W.skyjepa(seed=51, batch=B, samples=S, horizon=T, config=L.SkyJepaConfig.paper())
    H = w.model.history_steps
    doms, d_dom = _domains(B, 9)
    dom0 = L.Domain.default()
    high = float(np.float32(dom0.mass) * np.float32(dom0.gravity) * np.float32(dom0.max_thrust_weight) / 4)
    hover = np.float32(dom0.mass) * np.float32(dom0.gravity) / np.float32(4.0)
    cfg = L.MppiConfig(horizon=T, samples=S, action_dim=4, iterations=1,
                       action_bounds=L.ActionBounds.scalar(4, 0.0, high),
                       noise_std_per_action=[0.6, 0.15, 0.15, 0.05], temperature=1.0, seed=11)
    x0 = np.stack([L.hover_state() for _ in range(B)])
    x0[:, :3] += np.random.default_rng(3).uniform(-0.2, 0.2, (B, 3)).astype(np.float32)
    sh0 = np.repeat(x0[:, None], H, 1).astype(np.float32)
    ah0 = np.full((B, H - 1, 4), hover, np.float32)
    sc = L.SkyJepaScorer(ctx, w.model, w.weights, w.state_mean, w.state_std, w.action_mean, w.action_std, w.cost,
                         w.dt)
    sc.set_context(sh0, ah0, np.zeros((B, T, 18), np.float32), np.zeros((B, T, 4), np.float32))
    p_sh, p_ah, p_rs, p_ra = sc.context_device()
    view = lambda ptr, shape: L.device_tensor(ptr, shape)
    planner = L.MppiPlanner(ctx, cfg)
    d_x = _dev(x0)
    d_m = _dev(np.stack([np.full(4, d.mass * d.gravity / 4, np.float32) for d in doms]))
    # the oracle loop
    m = O.SkyJepaModel(w.model, w.weights)
    norm = (w.state_mean, w.state_std, w.action_mean, w.action_std)
    r_x, r_m = x0.copy(), np.stack([np.full(4, d.mass * d.gravity / 4, np.float32) for d in doms])
    r_sh, r_ah = sh0.copy(), ah0.copy()
    last = None
    per = S * T * 4 * B
    for k in range(steps):
        st = L.FleetStep()
        st.batch, st.horizon, st.history, st.time, st.dt = B, T, H, 0.05 * k, 0.05
        st.reference_kind, st.radius, st.period = 2, 2.0, 8.0
        st.prior_domain = dom0
        st.trim, st.state = None, d_x.data_ptr()
        st.last_action, st.last_action_stride = (last, 4) if last else (None, 4)
        st.state_history, st.action_history, st.reference_states, st.reference_actions = p_sh, p_ah, p_rs, p_ra
        L.fleet_control_step_device(ctx, st)
        planner.set_warm_start_device(p_ra, B)
        res = planner.plan_device(sc)
        L.plant_step_device(ctx, d_dom.data_ptr(), d_x.data_ptr(), d_m.data_ptr(), res.first_action, 4, B, 0.005, 10)
        last = res.first_action
        ctx.synchronize()
        got_seq = view(res.sequence, (B, T, 4)).cpu().numpy()
        # oracle: the same step from the same state (the GPU's), so states never drift apart
        if k > 0:
            r_sh = np.concatenate([r_sh[:, 1:], r_x[:, None]], 1)
            r_ah = np.concatenate([r_ah[:, 1:], r_last[:, None]], 1)
        refs = np.stack([O.reference_horizon(2, 0.05 * k, 0.05, T, 2.0, 8.0)] * B)
        prior = np.stack([np.clip(O.geometric_prior(r_x[b], refs[b], 0.05), 0.0, high) for b in range(B)])
        c = m.score_ctx(norm, r_sh, r_ah, refs, prior.astype(np.float32), w.cost, w.dt)
        ref = O.mppi_plan(cfg, B, (O.SKYJEPA_FN, c), seed=11, offset=k * (per + per % 2), warm_start=prior)
        assert_actions_close(got_seq, ref["sequence"])
        r_last = got_seq[:, 0].copy()
        for b in range(B):
            for _ in range(10):
                O.plant_step(doms[b], r_x[b], r_m[b], r_last[b], 0.005)
        np.testing.assert_allclose(d_x.cpu().numpy(), r_x, rtol=1e-4, atol=1e-4)
        r_x = d_x.cpu().numpy().copy()
        r_m = d_m.cpu().numpy().copy()
    planner.close()
    sc.close()
