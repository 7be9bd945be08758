"""The LeWM scorer with its GEMMs on the tensor cores (bf16 weights and GEMM
inputs, f32 accumulation; lwm_scorer_lewm_set_precision) against the f32
oracle, within the bf16 predictor tolerance of 2e-2 relative per candidate
cost."""
import numpy as np
import pytest

import lewm_b200 as L
import oracle as O
from gpu_helpers import normals
from lewm_b200 import workloads as W
from test_gpu_lewm import _score

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

BF16_REL = 2e-2


def _rel_norm(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return np.linalg.norm(got - ref) / np.linalg.norm(ref)


def assert_bf16_costs(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    err = np.abs(got - ref) / np.maximum(np.abs(ref), 1e-6)
    assert err.max() <= BF16_REL, f"worst relative cost error {err.max():.3g} at {np.unravel_index(err.argmax(), err.shape)}"


def test_vector_bf16_encoder_and_scores(ctx):
    w = W.lewm_vector(seed=21, batch=2)
    m = O.LewmModel(w.config, w.weights)
    sc = L.LewmScorer(ctx, w.config, w.weights)
    sc.set_precision("bf16")
    with torch.cuda.stream(ctx.torch_stream()):
        emb = sc.encode_vector(torch.as_tensor(w.obs).cuda())
    ctx.synchronize()
    assert _rel_norm(emb.cpu().numpy(), m.encode_vector(w.obs)) < BF16_REL
    # scores from the oracle's f32 context, so only the rollout differs
    e, g = m.encode_vector(w.obs)[:, None, :], m.encode_vector(w.goal_obs)
    sc.set_context(e, g)
    cand = np.clip(normals(61, (2, 300, 5, 2)), -1, 1).astype(np.float32)
    got = _score(ctx, sc, cand)
    assert_bf16_costs(got, m.scores(e, g, cand))
    # the tensor-core path is the one that ran: not bit-equal to the f32 GEMMs
    sc.set_precision("f32")
    f32 = _score(ctx, sc, cand)
    assert not np.array_equal(got, f32)
    sc.set_precision("bf16")
    assert np.array_equal(_score(ctx, sc, cand), got)  # deterministic (split-K in fixed order)


def test_image_bf16_pipeline(ctx):
    # the c4 model in bf16: ViT-Tiny encoder + projector, 6-layer predictor
    w = W.lewm_image(seed=22, samples=128)
    m = O.LewmModel(w.config, w.weights)
    sc = L.LewmScorer(ctx, w.config, w.weights)
    sc.set_precision("bf16")
    pix = np.random.default_rng(3).standard_normal((2, 3, 224, 224)).astype(np.float32)
    with torch.cuda.stream(ctx.torch_stream()):
        emb = sc.encode_pixels(torch.as_tensor(pix).cuda())
    ctx.synchronize()
    ref_emb = m.encode_pixels(pix)
    assert _rel_norm(emb.cpu().numpy(), ref_emb) < 3e-2
    e, g = ref_emb[:1, None, :], ref_emb[1:]
    sc.set_context(e, g)
    cand = np.clip(normals(62, (1, 128, 10, 2)), -1, 1).astype(np.float32)
    assert_bf16_costs(_score(ctx, sc, cand), m.scores(e, g, cand))


@pytest.mark.parametrize("S,T", [(37, 3), (1, 4), (130, 5)])
def test_ragged_tiles_and_history(ctx, S, T):
    # M not a multiple of 128 (and tiny); a 3-frame window with attention
    from test_lewm_oracle import small_config
    cfg = small_config(history=3)
    wts = cfg.random_weights(23)
    m = O.LewmModel(cfg, wts)
    sc = L.LewmScorer(ctx, cfg, wts)
    sc.set_precision("bf16")
    rng = np.random.default_rng(S)
    emb = rng.standard_normal((2, 3, cfg.embed_dim)).astype(np.float32)
    goal = rng.standard_normal((2, cfg.embed_dim)).astype(np.float32)
    sc.set_context(emb, goal)
    cand = rng.uniform(-1, 1, (2, S, T, 2)).astype(np.float32)
    assert_bf16_costs(_score(ctx, sc, cand), m.scores(emb, goal, cand))


def test_bf16_mppi_plan(ctx):
    w = W.lewm_vector(seed=24)
    m = O.LewmModel(w.config, w.weights)
    e, g = m.encode_vector(w.obs)[:, None, :], m.encode_vector(w.goal_obs)
    sc = L.LewmScorer(ctx, w.config, w.weights)
    sc.set_precision("bf16")
    sc.set_context(e, g)
    cfg = L.MppiConfig(horizon=5, samples=256, action_dim=2, iterations=1,
                       action_bounds=L.ActionBounds.symmetric(2, 1.0), noise_std=1.0, temperature=0.5)
    noise = normals(63, (1, 1, 256, 5, 2))
    r = L.MppiPlanner(ctx, cfg).plan(sc, injected_noise=noise)
    ref = O.mppi_plan(cfg, 1, (O.LEWM_FN, m.score_ctx(e, g)), noise=noise)
    assert_bf16_costs(r.scores, ref["scores"])
