"""The LeWM / WorldModel scorer on the GPU against the oracle
(LeWmSession::score_candidates, src/session.rs:46-66; modules.rs, vit.rs;
WorldModel::encode_vector, world_model/model.rs:207-274)."""
import numpy as np
import pytest

import lewm_b200 as L
import oracle as O
from gpu_helpers import assert_actions_close, assert_costs_close, assert_same_elites, normals
from lewm_b200 import workloads as W
from test_lewm_oracle import small_config, small_vit

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _score(ctx, sc, cand):
    B, S, T, A = cand.shape
    d = torch.as_tensor(cand).cuda()
    out = torch.empty((B, S), device="cuda")
    torch.cuda.synchronize()
    sc.score_device(d.data_ptr(), B, S, T, A, out.data_ptr())
    ctx.synchronize()
    return out.cpu().numpy()


def _vector_context(ctx, w):
    sc = L.LewmScorer(ctx, w.config, w.weights)
    with torch.cuda.stream(ctx.torch_stream()):
        emb = sc.encode_vector(torch.as_tensor(w.obs).cuda())
        goal = sc.encode_vector(torch.as_tensor(w.goal_obs).cuda())
    ctx.synchronize()
    return sc, emb, goal


def test_vector_encoder_matches_oracle(ctx):
    w = W.lewm_vector(seed=1, batch=3)
    sc, emb, goal = _vector_context(ctx, w)
    m = O.LewmModel(w.config, w.weights)
    np.testing.assert_allclose(emb.cpu().numpy(), m.encode_vector(w.obs), rtol=1e-4, atol=1e-4)


def test_vector_scores_match_oracle(ctx):
    w = W.lewm_vector(seed=2, batch=2)
    sc, emb, goal = _vector_context(ctx, w)
    sc.set_context_device(emb[:, None, :].contiguous(), goal)
    cand = np.clip(normals(51, (2, 300, 5, 2)), -1, 1).astype(np.float32)
    got = _score(ctx, sc, cand)
    m = O.LewmModel(w.config, w.weights)
    ref = m.scores(emb.cpu().numpy()[:, None, :], goal.cpu().numpy(), cand)
    assert_costs_close(got, ref)


@pytest.mark.parametrize("h, T", [(3, 6), (2, 2), (1, 4)])
def test_history_window_attention_matches_oracle(ctx, h, T):
    cfg = small_config(history=3)
    wts = cfg.random_weights(9)
    sc = L.LewmScorer(ctx, cfg, wts)
    rng = np.random.default_rng(h)
    emb = rng.standard_normal((2, h, cfg.embed_dim)).astype(np.float32)
    goal = rng.standard_normal((2, cfg.embed_dim)).astype(np.float32)
    sc.set_context(emb, goal)
    cand = rng.uniform(-1, 1, (2, 37, T, 2)).astype(np.float32)
    got = _score(ctx, sc, cand)
    ref = O.LewmModel(cfg, wts).scores(emb, goal, cand)
    assert_costs_close(got, ref)


def test_vector_cem_matches_oracle(ctx):
    # c3: 300 x 5, 30 elites, 3 iterations (CemPlanner::plan_device, src/planner.rs:450-541)
    w = W.lewm_vector(seed=3)
    sc, emb, goal = _vector_context(ctx, w)
    e, g = emb.cpu().numpy()[:, None, :], goal.cpu().numpy()
    sc.set_context(e, g)
    noise = normals(53, (3, 1, 300, 5, 2))
    planner = L.CemPlanner(ctx, w.planner)
    r = planner.plan(sc, injected_noise=noise)
    m = O.LewmModel(w.config, w.weights)
    ref = O.cem_plan(w.planner, 1, (O.LEWM_FN, m.score_ctx(e, g)), noise=noise)
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"])
    # the 30 elites of each of the 3 iterations equal the oracle's, up to ties within tolerance
    assert assert_same_elites(planner.elite_indices(), ref["elites"], ref["iteration_scores"]) >= 1


def test_small_vit_encoder_matches_oracle(ctx):
    cfg = small_vit()
    wts = cfg.random_weights(10)
    sc = L.LewmScorer(ctx, cfg, wts)
    pix = np.random.default_rng(5).standard_normal((3, 3, 32, 32)).astype(np.float32)
    with torch.cuda.stream(ctx.torch_stream()):
        out = sc.encode_pixels(torch.as_tensor(pix).cuda())
    ctx.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), O.LewmModel(cfg, wts).encode_pixels(pix), rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("image,patch", [(64, 8), (128, 8)])
def test_long_sequence_vit_attention_matches_oracle(ctx, image, patch):
    # 65 and 257 tokens: the shared-memory attention kernel (> 32 tokens; 257
    # exceeds its 256-token bound and takes the warp-per-query kernel)
    cfg = small_vit()
    cfg.image_size, cfg.patch_size = image, patch
    wts = cfg.random_weights(12)
    sc = L.LewmScorer(ctx, cfg, wts)
    pix = np.random.default_rng(6).standard_normal((2, 3, image, image)).astype(np.float32)
    with torch.cuda.stream(ctx.torch_stream()):
        out = sc.encode_pixels(torch.as_tensor(pix).cuda())
    ctx.synchronize()
    np.testing.assert_allclose(out.cpu().numpy(), O.LewmModel(cfg, wts).encode_pixels(pix), rtol=1e-4, atol=1e-4)


def test_image_pipeline_matches_oracle(ctx):
    # c4 model in f32: NV12 -> preprocess -> ViT-Tiny -> projector; then 64 candidates x 10 steps
    w = W.lewm_image(seed=4, samples=64)
    sc = L.LewmScorer(ctx, w.config, w.weights)
    cfg = L.ImagePreprocess.imagenet_224()
    pix = torch.empty((2, 3, 224, 224), device="cuda")
    y = torch.as_tensor(np.concatenate([w.y_plane, w.goal_y])).cuda()
    uv = torch.as_tensor(np.concatenate([w.uv_plane, w.goal_uv])).cuda()
    torch.cuda.synchronize()
    L.preprocess_nv12_device(ctx, y, uv, 2, 224, 224, "bt601-video", cfg, pix)
    with torch.cuda.stream(ctx.torch_stream()):
        emb = sc.encode_pixels(pix)
    ctx.synchronize()
    pix_ref = O.preprocess_nv12(np.concatenate([w.y_plane, w.goal_y]), np.concatenate([w.uv_plane, w.goal_uv]), 0,
                                224, 224, mean=cfg.mean[:], std=cfg.std[:])
    m = O.LewmModel(w.config, w.weights)
    emb_ref = m.encode_pixels(pix_ref)
    np.testing.assert_allclose(emb.cpu().numpy(), emb_ref, rtol=1e-3, atol=1e-3)
    sc.set_context_device(emb[:1, None, :].contiguous(), emb[1:].contiguous())
    cand = np.clip(normals(55, (1, 64, 10, 2)), -1, 1).astype(np.float32)
    got = _score(ctx, sc, cand)
    ref = m.scores(emb.cpu().numpy()[:1, None, :], emb.cpu().numpy()[1:], cand)
    assert_costs_close(got, ref)


@pytest.mark.parametrize("precision", ["f32", "bf16"])
def test_fused_frame_encoding_equals_preprocess_then_encode(ctx, precision):
    # the fused path (preprocess straight into the ViT patch matrix) feeds the
    # encoder the same values as preprocess -> NCHW -> patchify: identical
    # embeddings, with one launch fewer and no NCHW image
    w = W.lewm_image(seed=4, samples=64)
    sc = L.LewmScorer(ctx, w.config, w.weights)
    sc.set_precision(precision)
    cfg = L.ImagePreprocess.imagenet_224()
    y = torch.as_tensor(np.concatenate([w.y_plane, w.goal_y])).cuda()
    uv = torch.as_tensor(np.concatenate([w.uv_plane, w.goal_uv])).cuda()
    pix = torch.empty((2, 3, 224, 224), device="cuda")
    torch.cuda.synchronize()
    n0 = ctx.launch_count()
    L.preprocess_nv12_device(ctx, y, uv, 2, 224, 224, "bt601-video", cfg, pix)
    with torch.cuda.stream(ctx.torch_stream()):
        two_step = sc.encode_pixels(pix)
    ctx.synchronize()
    n1 = ctx.launch_count()
    with torch.cuda.stream(ctx.torch_stream()):
        fused = sc.encode_nv12(y, uv, 2, 224, 224, "bt601-video", cfg)
    ctx.synchronize()
    n2 = ctx.launch_count()
    assert torch.equal(fused, two_step)
    assert (n2 - n1) == (n1 - n0) - 1, "the fused path should save the patchify launch"
    # packed RGB frames through the same fused path
    rgb = np.random.default_rng(9).integers(0, 256, (2, 240, 320, 3), dtype=np.uint8)
    rgb_dev = torch.as_tensor(rgb).cuda()
    torch.cuda.synchronize()
    L.preprocess_packed_device(ctx, rgb_dev, 2, 240, 320, "rgb", cfg, pix)
    with torch.cuda.stream(ctx.torch_stream()):
        ref = sc.encode_pixels(pix)
        got = sc.encode_packed(rgb_dev, 2, 240, 320, "rgb", cfg)
    ctx.synchronize()
    assert torch.equal(got, ref)


def test_lewm_validation(ctx):
    cfg = L.LewmConfig.vector()
    with pytest.raises(L.LwmError, match="weight blob"):
        L.LewmScorer(ctx, cfg, np.zeros(10, np.float32))
    sc = L.LewmScorer(ctx, cfg, cfg.random_weights(1))
    with pytest.raises(L.LwmError, match="exceeds predictor.num_frames"):
        sc.set_context(np.zeros((1, 2, 192), np.float32), np.zeros((1, 192), np.float32))
    sc.set_context(np.zeros((1, 1, 192), np.float32), np.zeros((1, 192), np.float32))
    with pytest.raises(L.LwmError, match="do not match"):
        _score(ctx, sc, np.zeros((1, 4, 5, 3), np.float32))


def test_vector_mppi_matches_oracle(ctx):
    # MPPI over the LeWM scorer takes the generic sample -> score -> reduce path
    w = W.lewm_vector(seed=12)
    sc, emb, goal = _vector_context(ctx, w)
    e, g = emb.cpu().numpy()[:, None, :], goal.cpu().numpy()
    sc.set_context(e, g)
    cfg = L.MppiConfig(horizon=5, samples=256, action_dim=2, iterations=2,
                       action_bounds=L.ActionBounds.symmetric(2, 1.0), noise_std=1.0, temperature=0.5)
    noise = normals(57, (2, 1, 256, 5, 2))
    r = L.MppiPlanner(ctx, cfg).plan(sc, injected_noise=noise)
    m = O.LewmModel(w.config, w.weights)
    ref = O.mppi_plan(cfg, 1, (O.LEWM_FN, m.score_ctx(e, g)), noise=noise)
    assert_costs_close(r.scores, ref["scores"])
    assert_actions_close(r.sequence, ref["sequence"])
