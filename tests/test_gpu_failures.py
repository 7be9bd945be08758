"""Failure paths on the GPU, made to happen from the host.

The reference's only failure path is the planning deadline
(src/planner.rs:1055-1150, tested in test_gpu_planner.py).  Every pipeline
wait in this library's kernels is bounded; here a wait is made to run out on
purpose through lwm_ctx_set_test_faults — a hand-off that one warp skips (the
tensor-core rollout) or a source-row copy that the producer skips (row-staged
preprocessing) — with a short poll limit.  The kernel unwinds and returns
(nothing traps or hangs), the call reports the failure with the site, and
the next call on the same context gives the oracle's answer again."""
import zlib

import numpy as np
import pytest

import lewm_b200 as L
import oracle as O
from gpu_helpers import normals
from lewm_b200 import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

POLLS = 1 << 14  # a wait that gives up in well under a second


def _scorer(ctx, w):
    sc = L.SkyJepaScorer(ctx, w.model, w.weights, w.state_mean, w.state_std, w.action_mean, w.action_std, w.cost,
                         w.dt)
    sc.set_precision("bf16")
    sc.set_context(w.state_history, w.action_history, w.reference_states, w.reference_actions)
    return sc


def _oracle_scores(w, noise):
    m = O.SkyJepaModel(w.model, w.weights, tensor_core_rounding=True)
    c = m.score_ctx((w.state_mean, w.state_std, w.action_mean, w.action_std), w.state_history, w.action_history,
                    w.reference_states, w.reference_actions, w.cost, w.dt)
    return O.mppi_plan(w.mppi, w.batch, (O.SKYJEPA_FN, c), noise=noise, warm_start=w.warm_start)["scores"]


def test_tensor_core_wait_timeout_reports_and_recovers(ctx):
    w = W.skyjepa(seed=41, batch=2, samples=256, horizon=6)
    noise = normals(71, (1, 2, 256, 6, 4))
    planner = L.MppiPlanner(ctx, w.mppi)
    planner.set_warm_start_sequence(w.warm_start)
    sc = _scorer(ctx, w)
    ctx.set_test_faults(wait_polls=POLLS, tc_skip_h_arrive=True)
    try:
        with pytest.raises(L.LwmError) as e:
            planner.plan(sc, injected_noise=noise)
    finally:
        ctx.set_test_faults()
    # the first wait to give up records its site: the MMA issuer's wait for h
    # (site 2) or the weight producer's wait behind it (site 1), in block 0
    assert e.value.status == "TIMEOUT" and "block 0" in e.value.message, str(e.value)
    assert any(f"site {k}," in e.value.message for k in (1, 2)), str(e.value)
    # the context, the scorer and the planner keep working
    ref = _oracle_scores(w, noise)
    planner.set_warm_start_sequence(w.warm_start)
    r = planner.plan(sc, injected_noise=noise)
    rel = np.abs(np.asarray(r.scores, np.float64) - ref) / np.maximum(np.abs(ref), 1e-6)
    assert rel.max() <= 1e-4
    p2 = L.MppiPlanner(ctx, w.mppi)
    p2.set_warm_start_sequence(w.warm_start)
    r2 = p2.plan(_scorer(ctx, w), injected_noise=noise)
    assert np.array_equal(np.asarray(r2.scores), np.asarray(r.scores))
    assert np.array_equal(np.asarray(r2.sequence), np.asarray(r.sequence))


@pytest.mark.parametrize("fmt", ["nv12", "rgba"])
def test_preprocessing_wait_timeout_reports_and_recovers(ctx, fmt):
    B, H, W_, oh, ow = 2, 120, 160, 96, 128  # row-staged shapes
    rng = np.random.default_rng(zlib.crc32(fmt.encode()))
    cfg = L.ImagePreprocess.make(oh, ow, mean=(0.485, 0.456, 0.406), std=(0.229, 0.224, 0.225))
    out = torch.zeros((B, 3, oh, ow), device="cuda")
    if fmt == "nv12":
        y = rng.integers(0, 256, (B, H, W_), dtype=np.uint8)
        uv = rng.integers(0, 256, (B, H // 2, W_ // 2, 2), dtype=np.uint8)
        dy, duv = torch.from_numpy(y).cuda(), torch.from_numpy(uv).cuda()
        run = lambda: L.preprocess_nv12_device(ctx, dy, duv, B, H, W_, "bt601-video", cfg, out)  # noqa: E731
        ref = O.preprocess_nv12(y, uv, 0, oh, ow, mean=cfg.mean[:], std=cfg.std[:])
    else:
        frames = rng.integers(0, 256, (B, H, W_, 4), dtype=np.uint8)
        df = torch.from_numpy(frames).cuda()
        run = lambda: L.preprocess_packed_device(ctx, df, B, H, W_, "rgba", cfg, out)  # noqa: E731
        ref = O.preprocess_packed(frames, L.PACKED_FORMATS["rgba"], oh, ow, mean=cfg.mean[:], std=cfg.std[:])
    torch.cuda.synchronize()
    ctx.set_test_faults(wait_polls=POLLS, media_skip_row=37)
    try:
        run()
        with pytest.raises(L.LwmError) as e:
            ctx.synchronize()
    finally:
        ctx.set_test_faults()
    assert e.value.status == "CUDA_ERROR" and "never completed" in e.value.message, str(e.value)
    ctx.synchronize()  # reported once
    run()
    ctx.synchronize()
    assert np.array_equal(out.cpu().numpy(), ref)
