"""LeWM image control step in one call (lwm_lewm_plan_nv12_device): NV12
frames -> ViT embeddings -> scorer context -> MPPI plan, with the frames'
encoder on a second stream beside sampling and the candidate-only part of
scoring.  Held to the three-call path (encode_nv12, set_context_device,
plan_device) on the same frames and planner seed, over two plans in a row
(the second one warm-started).  The reference step is LeWmSession
(src/session.rs:31-65) under MppiPlanner::plan (src/planner.rs:446-450)."""

import numpy as np
import pytest

import lewm_b200 as L
from lewm_b200 import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _host(ctx, r, w):
    ctx.synchronize()  # the context stream does not synchronise with torch's default stream
    B, T, A = w.batch, w.horizon, w.config.action_dim
    seq = L.device_tensor(r.sequence, (B, T, A)).cpu().numpy()
    scores = L.device_tensor(r.scores, (B, r.scores_cols)).cpu().numpy()
    best = L.device_tensor(r.best_indices, (B,), "u4").cpu().numpy()
    return seq, scores, best


def _frames(w, step):
    # step 1 swaps observation and goal, so both plans see new context
    obs_y, obs_uv, goal_y, goal_uv = w.y_plane, w.uv_plane, w.goal_y, w.goal_uv
    if step == 1:
        obs_y, obs_uv, goal_y, goal_uv = goal_y, goal_uv, obs_y, obs_uv
    y = torch.from_numpy(np.concatenate([obs_y, goal_y])).cuda()
    uv = torch.from_numpy(np.concatenate([obs_uv, goal_uv])).cuda()
    return y, uv


@pytest.mark.parametrize("batch,samples", [(1, 1024), (2, 128)])
def test_plan_nv12_matches_encode_then_plan(ctx, batch, samples):
    # the same kernels on the same inputs in the same summation order (the
    # candidate-only part has its own split-K scratch): bit-equal results;
    # 128 samples split K for the action embedder's last layer, 1024 do not
    w = W.lewm_image(seed=41, batch=batch, samples=samples)
    prep = L.ImagePreprocess.imagenet_224()
    s = w.config.image_size
    sc = L.LewmScorer(ctx, w.config, w.weights)
    sc.set_precision("bf16")
    three, one = L.MppiPlanner(ctx, w.planner), L.MppiPlanner(ctx, w.planner)
    stream = ctx.torch_stream()
    for step in range(2):
        with torch.cuda.stream(stream):
            y, uv = _frames(w, step)
            emb = sc.encode_nv12(y, uv, 2 * batch, s, s, "bt601-video", prep)
            sc.set_context_device(emb[:batch, None, :].contiguous(), emb[batch:].contiguous())
        ref = _host(ctx, three.plan_device(sc), w)
        with torch.cuda.stream(stream):
            y, uv = _frames(w, step)
        got = _host(ctx, one.plan_nv12_device(sc, y, uv, batch, 1, s, s, "bt601-video", prep), w)
        for g, r in zip(got, ref):
            np.testing.assert_array_equal(g, r)


def test_plan_nv12_rejects_bad_arguments(ctx):
    w = W.lewm_image(seed=42, samples=64)
    s = w.config.image_size
    sc = L.LewmScorer(ctx, w.config, w.weights)
    planner = L.MppiPlanner(ctx, w.planner)
    y, uv = _frames(w, 0)
    small = L.ImagePreprocess.imagenet_224()
    small.output_height = small.output_width = 112
    with pytest.raises(L.LwmError, match="does not match the encoder's image size"):
        planner.plan_nv12_device(sc, y, uv, 1, 1, s, s, "bt601-video", small)
    with pytest.raises(L.LwmError, match="exceeds predictor.num_frames"):
        planner.plan_nv12_device(sc, y, uv, 1, 2, s, s, "bt601-video", L.ImagePreprocess.imagenet_224())
