"""Planner pieces and planners on the GPU, through the C ABI, against the
oracle and the reference's planner unit tests (src/planner.rs:1898-2158)."""
import numpy as np
import pytest

import lewm_b200 as L
import oracle as O
from gpu_helpers import assert_actions_close, assert_same_elites, normals

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _dev(a, dtype=torch.float32):
    return torch.as_tensor(np.ascontiguousarray(a)).to(device="cuda", dtype=dtype)


def test_normals_match_oracle(ctx):
    n = 1 << 16
    out = torch.empty(n, device="cuda")
    torch.cuda.synchronize()
    L.normal_device(ctx, 77, 12345, n, out.data_ptr())
    ctx.synchronize()
    ref = O.normals(77, 12345, n)
    got = out.cpu().numpy()
    assert np.abs(got - ref).max() < 2e-5 * max(1.0, np.abs(ref).max())


def _lowest_k(ctx, scores, k):
    s = _dev(scores)
    B, S = scores.shape
    out = torch.empty((B, k), dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    L.lowest_k_device(ctx, s.data_ptr(), B, S, k, out.data_ptr())
    ctx.synchronize()
    return out.cpu().numpy().astype(np.uint32)


def test_lowest_k_reference_known_answers(ctx):
    # src/planner.rs:1922-1941
    assert _lowest_k(ctx, np.array([[3, 1, 4, 0.5], [9, -1, 2, -2]], np.float32), 3).tolist() == [[3, 1, 0], [3, 1, 2]]
    desc = np.array([[1024 - i for i in range(1024)]], np.float32)
    assert _lowest_k(ctx, desc, 4).tolist() == [[1023, 1022, 1021, 1020]]
    weird = np.array([[np.nan, 2.0, 1.0, 1.0, -0.0, 0.0, np.inf]], np.float32)
    assert _lowest_k(ctx, weird, 7).tolist() == O.lowest_k(weird, 7).tolist()


# Rows up to 4096 scores are sorted whole; longer ones go through the radix
# selection (no limit on the row length), including K = S and K at its limit.
@pytest.mark.parametrize("S,k", [(1, 1), (7, 3), (300, 30), (4096, 64), (4097, 4097), (5000, 17), (16384, 100),
                                 (20000, 16384), (65536, 30), (100003, 4096)])
def test_lowest_k_bit_exact_with_ties(ctx, S, k):
    rng = np.random.default_rng(S)
    scores = rng.integers(0, max(2, S // 8), (3, S)).astype(np.float32)  # many ties
    scores[0, rng.integers(0, S, max(1, S // 50))] = np.nan
    scores[2] = rng.standard_normal(S).astype(np.float32)                # distinct values
    assert np.array_equal(_lowest_k(ctx, scores, k), O.lowest_k(scores, k))


def test_lowest_k_selection_degenerate_rows(ctx):
    # every score tied, all NaN, +-inf only, NaN with three finite values at
    # the end, signed zeros: the selection path orders them as the full sort
    S = 9000
    idx = np.arange(S)
    rows = np.stack([np.full(S, np.nan), np.full(S, 1.5), np.where(idx % 2 == 1, np.inf, -np.inf),
                     np.concatenate([np.full(S - 3, np.nan), [3.0, 2.0, 1.0]]),
                     np.where(idx % 3 == 0, -0.0, 0.0)]).astype(np.float32)
    for k in (1, 5, 4500, S):
        assert np.array_equal(_lowest_k(ctx, rows, min(k, 16384)), O.lowest_k(rows, min(k, 16384))), k


def test_lowest_k_rejects_more_than_its_elite_limit(ctx):
    s = torch.zeros((1, 20000), device="cuda")
    out = torch.empty((1, 16385), dtype=torch.int32, device="cuda")
    with pytest.raises(L.LwmError, match="at most 16384"):
        L.lowest_k_device(ctx, s.data_ptr(), 1, 20000, 16385, out.data_ptr())


def test_cem_beyond_sixteen_thousand_samples_matches_oracle(ctx):
    # the reference has no sample limit (arg-sort fallback, src/planner.rs:1655-1658)
    cfg = L.CemConfig(horizon=4, samples=40000, elites=64, action_dim=2, iterations=2, init_std=0.8, seed=8)
    noise = normals(14, (2, 1, 40000, 4, 2))
    target = [0.3, -0.2]
    planner = L.CemPlanner(ctx, cfg)
    r = planner.plan(L.CallbackScorer(ctx, 1, _quad(target)), injected_noise=noise)
    ref = O.cem_plan(cfg, 1, lambda c: ((c - np.array(target, np.float32)) ** 2).sum(axis=(2, 3)), noise=noise)
    assert_actions_close(r.sequence, ref["sequence"], 1e-5)
    assert r.best_indices == ref["best"].tolist()
    assert assert_same_elites(planner.elite_indices(), ref["elites"], ref["iteration_scores"], rel=1e-6) == 2


def test_lowest_k_rejects_count_above_samples(ctx):
    s = torch.zeros((1, 4), device="cuda")
    out = torch.empty((1, 5), dtype=torch.int32, device="cuda")
    with pytest.raises(L.LwmError, match="top-k count 5 cannot exceed samples 4"):
        L.lowest_k_device(ctx, s.data_ptr(), 1, 4, 5, out.data_ptr())


def test_color_noise_matches_oracle(ctx):
    noise = normals(3, (2, 8, 6, 4))
    d = _dev(noise)
    out = torch.empty_like(d)
    torch.cuda.synchronize()
    L.color_noise_device(ctx, d.data_ptr(), out.data_ptr(), 2, 8, 6, 4, 2.0)
    ctx.synchronize()
    got = out.cpu().numpy()
    assert np.isfinite(got).all()
    assert np.abs(got - O.color_noise(noise, 2.0)).max() < 1e-5


def _sum_scorer(c):
    return (c ** 2).sum(dim=(2, 3))


def test_mppi_uses_per_action_noise_and_shifts_warm_start(ctx):
    # src/planner.rs:2094-2137
    cfg = L.MppiConfig(horizon=3, samples=1, action_dim=2, noise_std_per_action=[0.6, 0.1], seed=9)
    planner = L.MppiPlanner(ctx, cfg)
    initial = np.array([[[0.1, 0.2], [0.3, 0.4], [0.5, 0.6]]], np.float32)
    planner.set_warm_start_sequence(initial)
    r = planner.plan(L.CallbackScorer(ctx, 1, _sum_scorer))
    assert np.array_equal(r.sequence, initial)
    assert np.array_equal(planner.warm_start_sequence(), np.array([[[0.3, 0.4], [0.5, 0.6], [0.5, 0.6]]], np.float32))


def _fixed(c):
    B, S = c.shape[:2]
    s = torch.arange(S, dtype=torch.float32, device=c.device).repeat(B, 1)
    s[:, 0] = 100.0
    return s


@pytest.mark.parametrize("return_mean", [True, False])
def test_icem_fixed_score_reference_tests(ctx, return_mean):
    # src/planner.rs:1997-2092
    cfg = L.IcemConfig(horizon=2, samples=4, elites=2, action_dim=1, iterations=1, keep_elites=0, alpha=1.0,
                       init_std=0.5, seed=123, return_mean=return_mean)
    planner = L.IcemPlanner(ctx, cfg)
    warm = np.array([[[0.25], [-0.5]]], np.float32)
    planner.set_warm_start_sequence(warm)
    r = planner.plan(L.CallbackScorer(ctx, 1, _fixed))
    assert r.best_indices == [1]
    assert np.array_equal(r.sequence, warm) == return_mean


def _quad(target):
    t = torch.tensor(target, device="cuda", dtype=torch.float32)
    return lambda c: ((c - t) ** 2).sum(dim=(2, 3))


def test_cem_matches_oracle_with_injected_noise(ctx):
    cfg = L.CemConfig(horizon=5, samples=300, elites=30, action_dim=2, iterations=3, seed=4)
    B = 2
    noise = normals(9, (3, B, 300, 5, 2))
    target = [0.3, -0.4]
    r = L.CemPlanner(ctx, cfg).plan(L.CallbackScorer(ctx, B, _quad(target)), injected_noise=noise)
    ref = O.cem_plan(cfg, B, lambda c: ((c - np.array(target, np.float32)) ** 2).sum(axis=(2, 3)), noise=noise)
    assert_actions_close(r.sequence, ref["sequence"], 1e-5)
    assert np.abs(r.scores - ref["scores"]).max() < 1e-4
    assert r.best_indices == ref["best"].tolist()


def test_icem_matches_oracle_with_colored_noise_and_carried_elites(ctx):
    cfg = L.IcemConfig(horizon=6, samples=64, elites=8, action_dim=3, keep_elites=3, iterations=3, noise_beta=2.0,
                       alpha=0.1, seed=5)
    noise = normals(10, (3, 1, 64, 6, 3))
    warm = normals(11, (1, 6, 3)) * 0.1
    target = [0.2, -0.1, 0.5]
    p = L.IcemPlanner(ctx, cfg)
    p.set_warm_start_sequence(warm)
    r = p.plan(L.CallbackScorer(ctx, 1, _quad(target)), injected_noise=noise)
    ref = O.icem_plan(cfg, 1, lambda c: ((c - np.array(target, np.float32)) ** 2).sum(axis=(2, 3)), noise=noise,
                      warm_start=warm)
    assert_actions_close(r.sequence, ref["sequence"], 1e-5)
    assert r.best_indices == ref["best"].tolist()
    assert_actions_close(p.warm_start_sequence(), ref["warm"], 1e-5)
    assert assert_same_elites(p.elite_indices(), ref["elites"], ref["iteration_scores"]) == 3


def test_mppi_generic_matches_oracle(ctx):
    cfg = L.MppiConfig(horizon=8, samples=1000, action_dim=2, iterations=2, temperature=0.5, seed=6)
    noise = normals(12, (2, 1, 1000, 8, 2))
    target = [0.5, 0.1]
    r = L.MppiPlanner(ctx, cfg).plan(L.CallbackScorer(ctx, 1, _quad(target)), injected_noise=noise)
    ref = O.mppi_plan(cfg, 1, lambda c: ((c - np.array(target, np.float32)) ** 2).sum(axis=(2, 3)), noise=noise)
    assert_actions_close(r.sequence, ref["sequence"], 1e-5)
    assert r.best_indices == ref["best"].tolist()


def test_seeded_planner_reserves_draws_and_resets(ctx):
    # PlannerRng (src/planner.rs:1380-1423, 1488-1514)
    cfg = L.MppiConfig(horizon=3, samples=5, action_dim=3, iterations=2, seed=21)
    p = L.MppiPlanner(ctx, cfg)
    sc = L.CallbackScorer(ctx, 1, _sum_scorer)
    a = p.plan(sc)
    assert p.rng_offset() == 46 * 2  # round_even(1*5*3*3 = 45) = 46 per iteration
    p.reset_rng_sequence()
    p.clear_warm_start()
    assert p.rng_offset() == 0
    b = p.plan(sc)
    assert np.array_equal(a.sequence, b.sequence)


def test_deadline_outcomes(ctx):
    # src/planner.rs:629-653, 1090-1150
    sc = L.CallbackScorer(ctx, 1, _sum_scorer)
    p = L.MppiPlanner(ctx, L.MppiConfig(horizon=3, samples=8, action_dim=2, deadline=0.0, deadline_action=[0.1, 0.2]))
    r = p.plan(sc)
    assert r.deadline_reached and r.deadline_outcome == "ConfiguredAction" and r.iterations_completed == 0
    assert np.array_equal(r.sequence, np.tile(np.array([0.1, 0.2], np.float32), (1, 3, 1)))
    assert r.scores.shape == (1, 1) and r.best_indices == [0]
    warm = np.full((1, 3, 2), 0.5, np.float32)
    p.set_warm_start_sequence(warm)
    r = p.plan(sc)
    assert r.deadline_outcome == "WarmStart" and np.array_equal(r.sequence, warm)
    p2 = L.MppiPlanner(ctx, L.MppiConfig(horizon=3, samples=8, action_dim=2, deadline=0.0))
    with pytest.raises(L.LwmError, match="MPPI deadline reached before any iteration completed and no "
                                         "deadline_action is configured"):
        p2.plan(sc)
    c = L.CemPlanner(ctx, L.CemConfig(horizon=3, samples=8, elites=2, action_dim=2, deadline=0.0))
    with pytest.raises(L.LwmError, match="CEM deadline reached"):
        c.plan(sc)


def test_warm_start_shape_mismatch_is_an_error(ctx):
    p = L.MppiPlanner(ctx, L.MppiConfig(horizon=3, samples=8, action_dim=2))
    p.set_warm_start_sequence(np.zeros((2, 3, 2), np.float32))
    with pytest.raises(L.LwmError, match=r"MPPI warm-start shape \[2, 3, 2\] does not match expected \[1, 3, 2\]"):
        p.plan(L.CallbackScorer(ctx, 1, _sum_scorer))


def test_icem_trace_matches_oracle(ctx):
    # IcemPlanner::trace_device (src/planner.rs:900-1010) with the fused nominal
    # scorer (the mean / elite-mean / updated-mean scores run it with one sample)
    from lewm_b200 import workloads as W
    w = W.nominal(seed=31, batch=2, samples=128, horizon=8)
    cfg = L.IcemConfig(horizon=8, samples=128, elites=12, action_dim=4, keep_elites=2, iterations=3,
                       noise_beta=1.5, alpha=0.1, init_std=0.5, action_bounds=w.mppi.action_bounds)
    noise = normals(33, (3, 2, 128, 8, 4))
    sc = L.NominalScorer(ctx, w.dt, w.trim, w.cost, w.substeps)
    sc.set_context(w.initial, w.motors, w.reference_states, w.reference_actions)
    p = L.IcemPlanner(ctx, cfg)
    p.set_warm_start_sequence(w.warm_start)
    d_noise = torch.as_tensor(noise).cuda()
    torch.cuda.synchronize()
    res, steps = p.trace_device(sc, d_noise.data_ptr())
    ctx.synchronize()
    seq = L.device_tensor(res.sequence, (2, 8, 4)).cpu().numpy()
    ref = O.icem_trace(cfg, 2, (O.NOMINAL_FN, O.nominal_ctx(w.initial, w.motors, w.reference_states,
                                                             w.reference_actions, w.cost, w.dt, w.trim)),
                       noise=noise, warm_start=w.warm_start)
    assert steps.shape == (3, 4, 2)
    assert_actions_close(seq, ref["sequence"])
    np.testing.assert_allclose(steps, ref["trace"], rtol=1e-4, atol=1e-5)


def test_icem_trace_with_callback_scorer(ctx):
    cfg = L.IcemConfig(horizon=6, samples=64, elites=8, action_dim=3, keep_elites=3, iterations=3, noise_beta=2.0,
                       alpha=0.1, seed=5)
    noise = normals(10, (3, 1, 64, 6, 3))
    warm = normals(11, (1, 6, 3)) * 0.1
    target = [0.2, -0.1, 0.5]
    p = L.IcemPlanner(ctx, cfg)
    p.set_warm_start_sequence(warm)
    d_noise = torch.as_tensor(noise).cuda()
    torch.cuda.synchronize()
    res, steps = p.trace_device(L.CallbackScorer(ctx, 1, _quad(target)), d_noise.data_ptr())
    ctx.synchronize()
    ref = O.icem_trace(cfg, 1, lambda c: ((c - np.array(target, np.float32)) ** 2).sum(axis=(2, 3)), noise=noise,
                       warm_start=warm)
    assert_actions_close(L.device_tensor(res.sequence, (1, 6, 3)).cpu().numpy(), ref["sequence"], 1e-5)
    np.testing.assert_allclose(steps, ref["trace"], rtol=1e-4, atol=1e-5)
    assert_actions_close(p.warm_start_sequence(), ref["warm"], 1e-5)
