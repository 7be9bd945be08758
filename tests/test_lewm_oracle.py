"""The LeWM / WorldModel oracle (oracle/lewm_world.c) without a GPU.

The reference's Candle modules cannot run here, so the oracle's restatement
of src/models/lewm/modules.rs, model.rs and vit.rs is cross-checked against
an independent torch (CPU, float64) implementation of the same published
operations, reading the same weight blob in the documented order:
AdaLN-conditioned causal transformer blocks, the action embedder, the MLP
heads (BatchNorm eval / LayerNorm), the vector encoder and a ViT.  Also
checked: the product's weight layout count equals the oracle's, and the
session scoring rule (src/session.rs:74-100): scoring with the session's
history equals a direct rollout with history = h."""
import ctypes as C

import numpy as np
import pytest

import lewm_b200 as L
import oracle as O

torch = pytest.importorskip("torch")
F = torch.nn.functional


class Blob:
    def __init__(self, w):
        self.w = torch.from_numpy(np.asarray(w, np.float64))
        self.off = 0

    def take(self, *shape):
        n = int(np.prod(shape))
        t = self.w[self.off:self.off + n].reshape(shape)
        self.off += n
        return t

    def lin(self, out, inp, bias=True):
        return (self.take(out, inp), self.take(out) if bias else None)

    def norm(self, kind, d):
        if kind == 0:
            return ("batch", self.take(d), self.take(d), self.take(d), self.take(d))
        if kind == 1:
            return ("layer", self.take(d), self.take(d))
        return ("none",)

    def mlp(self, inp, hid, out, kind):
        return (self.lin(hid, inp), self.norm(kind, hid), self.lin(out, hid))


def linear(x, l):
    w, b = l
    y = x @ w.T
    return y + b if b is not None else y


def norm_apply(x, n, eps=1e-5):
    if n[0] == "layer":
        return F.layer_norm(x, (x.shape[-1],), n[1], n[2], eps)
    if n[0] == "batch":
        return (x - n[3]) / torch.sqrt(n[4] + eps) * n[1] + n[2]
    return x


def mlp(x, m):
    return linear(F.gelu(norm_apply(linear(x, m[0]), m[1]), approximate="tanh"), m[2])


def parse(cfg, w):
    b = Blob(w)
    D, hid, inner = cfg.embed_dim, cfg.pred_hidden_dim, cfg.heads * cfg.dim_head
    p = {"act": (b.lin(cfg.smoothed_dim, cfg.action_dim), b.lin(cfg.action_mlp_scale * D, cfg.smoothed_dim),
                 b.lin(D, cfg.action_mlp_scale * D)),
         "pos": b.take(cfg.num_frames, D)}
    assert hid == D
    p["blocks"] = []
    for _ in range(cfg.depth):
        p["blocks"].append(dict(attn_norm=b.norm(1, hid), qkv=b.lin(3 * inner, hid, False), out=b.lin(hid, inner),
                                mlp_norm=b.norm(1, hid), fc1=b.lin(cfg.mlp_dim, hid), fc2=b.lin(hid, cfg.mlp_dim),
                                ada=b.lin(6 * hid, hid)))
    p["norm"] = b.norm(1, hid)
    p["pred_proj"] = b.mlp(D, cfg.pred_proj_hidden, D, cfg.pred_proj_norm)
    if cfg.encoder == 0:
        enc = []
        for j in range(cfg.obs_depth):
            inp = cfg.obs_dim if j == 0 else cfg.obs_hidden_dim
            out = D if j == cfg.obs_depth - 1 else cfg.obs_hidden_dim
            l = b.lin(out, inp)
            n = b.norm(1 if cfg.obs_norm != 2 else 2, cfg.obs_hidden_dim) if j + 1 < cfg.obs_depth else ("none",)
            enc.append((l, n))
        p["enc"] = enc
    else:
        vh, ps = cfg.vit_hidden, cfg.patch_size
        side = cfg.image_size // ps
        p["cls"] = b.take(vh)
        p["vpos"] = b.take(side * side + 1, vh)
        p["patch"] = b.lin(vh, cfg.channels * ps * ps)
        p["vit"] = []
        for _ in range(cfg.vit_layers):
            p["vit"].append(dict(ln1=b.norm(1, vh), q=b.lin(vh, vh, bool(cfg.qkv_bias)),
                                 k=b.lin(vh, vh, bool(cfg.qkv_bias)), v=b.lin(vh, vh, bool(cfg.qkv_bias)),
                                 o=b.lin(vh, vh), ln2=b.norm(1, vh), fc1=b.lin(cfg.vit_mlp, vh),
                                 fc2=b.lin(vh, cfg.vit_mlp)))
        p["vit_norm"] = b.norm(1, vh)
        p["projector"] = b.mlp(vh, cfg.projector_hidden, D, cfg.projector_norm)
    assert b.off == len(w)
    return p


def ln0(x, eps):
    return F.layer_norm(x, (x.shape[-1],), None, None, eps)


def predict_last(cfg, p, frames, act_emb):
    """Predictor::forward_last + pred_proj, in float64 torch."""
    x = frames + p["pos"][: frames.shape[1]]
    c = F.silu(act_emb)
    t = x.shape[1]
    H, dh = cfg.heads, cfg.dim_head
    mask = torch.full((t, t), float("-inf"), dtype=x.dtype).triu(1)
    for blk in p["blocks"]:
        sh1, sc1, g1, sh2, sc2, g2 = linear(c, blk["ada"]).chunk(6, -1)
        a = F.layer_norm(ln0(x, 1e-6) * (sc1 + 1) + sh1, (x.shape[-1],), blk["attn_norm"][1],
                         blk["attn_norm"][2], 1e-5)
        q, k, v = linear(a, blk["qkv"]).reshape(x.shape[0], t, 3, H, dh).permute(2, 0, 3, 1, 4)
        att = torch.softmax((q * dh ** -0.5) @ k.transpose(-1, -2) + mask, -1) @ v
        x = x + g1 * linear(att.permute(0, 2, 1, 3).reshape(x.shape[0], t, H * dh), blk["out"])
        m = F.layer_norm(ln0(x, 1e-6) * (sc2 + 1) + sh2, (x.shape[-1],), blk["mlp_norm"][1], blk["mlp_norm"][2],
                         1e-5)
        x = x + g2 * linear(F.gelu(linear(m, blk["fc1"]), approximate="tanh"), blk["fc2"])
    last = F.layer_norm(x[:, -1], (x.shape[-1],), p["norm"][1], p["norm"][2], 1e-5)
    return mlp(last, p["pred_proj"])


def action_embed(p, a):
    return linear(F.silu(linear(linear(a, p["act"][0]), p["act"][1])), p["act"][2])


def small_config(history=3):
    c = L.LewmConfig.vector()
    c.embed_dim = 64
    c.pred_hidden_dim = 64
    c.depth = 2
    c.heads = 4
    c.dim_head = 16
    c.mlp_dim = 96
    c.pred_proj_hidden = 80
    c.obs_hidden_dim = 48
    c.history_size = history
    c.num_frames = history
    return c


@pytest.mark.parametrize("make", [L.LewmConfig.vector, L.LewmConfig.image, small_config])
def test_weight_count_product_equals_oracle(make):
    cfg = make()
    assert cfg.weight_count() == O.lib.orc_lewm_weight_count(C.byref(cfg)) > 0


def test_presets_mirror_the_workload_models():
    v = L.LewmConfig.vector()
    assert (v.obs_dim, v.obs_hidden_dim, v.embed_dim, v.depth, v.heads, v.dim_head, v.mlp_dim) == \
        (16, 512, 192, 4, 8, 32, 768)
    i = L.LewmConfig.image()
    assert (i.image_size, i.patch_size, i.vit_layers, i.vit_hidden, i.vit_heads, i.vit_mlp) == (224, 16, 12, 192, 3, 768)
    assert (i.depth, i.heads, i.dim_head, i.mlp_dim, i.pred_proj_norm) == (6, 16, 64, 2048, 0)


@pytest.mark.parametrize("t", [1, 3])
def test_oracle_predictor_matches_torch(t):
    cfg = small_config(history=3)
    w = cfg.random_weights(5)
    m = O.LewmModel(cfg, w)
    p = parse(cfg, w)
    rng = np.random.default_rng(1)
    frames = rng.standard_normal((7, t, cfg.embed_dim)).astype(np.float32)
    acts = rng.uniform(-1, 1, (7, t, cfg.action_dim)).astype(np.float32)
    emb = m.action_embed(acts).reshape(7, t, -1)
    want_emb = action_embed(p, torch.from_numpy(acts).double()).numpy()
    np.testing.assert_allclose(emb, want_emb, rtol=2e-5, atol=2e-5)
    got = m.predict_last(frames, emb)
    want = predict_last(cfg, p, torch.from_numpy(frames).double(), torch.from_numpy(emb).double()).numpy()
    np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4)


def test_oracle_vector_encoder_matches_torch():
    cfg = L.LewmConfig.vector()
    w = cfg.random_weights(6)
    m = O.LewmModel(cfg, w)
    p = parse(cfg, w)
    obs = np.random.default_rng(2).standard_normal((5, 16)).astype(np.float32)
    x = torch.from_numpy(obs).double()
    for l, n in p["enc"][:-1]:
        x = F.gelu(norm_apply(linear(x, l), n), approximate="tanh")
    want = linear(x, p["enc"][-1][0]).numpy()
    np.testing.assert_allclose(m.encode_vector(obs), want, rtol=1e-4, atol=1e-4)


def small_vit():
    c = L.LewmConfig.image()
    c.image_size, c.patch_size, c.vit_hidden, c.vit_layers, c.vit_heads, c.vit_mlp = 32, 8, 48, 2, 3, 64
    c.projector_hidden = 40
    c.embed_dim = c.pred_hidden_dim = 32
    c.depth, c.heads, c.dim_head, c.mlp_dim, c.pred_proj_hidden = 1, 2, 16, 40, 24
    return c


def test_oracle_vit_matches_torch():
    cfg = small_vit()
    w = cfg.random_weights(7)
    m = O.LewmModel(cfg, w)
    p = parse(cfg, w)
    pix = np.random.default_rng(3).standard_normal((2, 3, 32, 32)).astype(np.float32)
    x = torch.from_numpy(pix).double()
    ps, vh = cfg.patch_size, cfg.vit_hidden
    wconv = p["patch"][0].reshape(vh, 3, ps, ps)
    e = F.conv2d(x, wconv, p["patch"][1], stride=ps).flatten(2).transpose(1, 2)
    tok = torch.cat([p["cls"].expand(2, 1, vh), e], 1) + p["vpos"]
    H = cfg.vit_heads
    dh = vh // H
    for blk in p["vit"]:
        a = F.layer_norm(tok, (vh,), blk["ln1"][1], blk["ln1"][2], cfg.vit_eps)
        sp = lambda t: t.reshape(2, -1, H, dh).transpose(1, 2)
        q, k, v = sp(linear(a, blk["q"])), sp(linear(a, blk["k"])), sp(linear(a, blk["v"]))
        att = torch.softmax(q @ k.transpose(-1, -2) / dh ** 0.5, -1) @ v
        tok = linear(att.transpose(1, 2).reshape(2, -1, vh), blk["o"]) + tok
        mm = F.layer_norm(tok, (vh,), blk["ln2"][1], blk["ln2"][2], cfg.vit_eps)
        tok = linear(F.gelu(linear(mm, blk["fc1"])), blk["fc2"]) + tok
    cls = F.layer_norm(tok, (vh,), p["vit_norm"][1], p["vit_norm"][2], cfg.vit_eps)[:, 0]
    want = mlp(cls, p["projector"]).numpy()
    np.testing.assert_allclose(m.encode_pixels(pix), want, rtol=1e-4, atol=1e-4)


def test_rollout_window_semantics():
    # rollout_embeddings_with_history (model.rs:94-147): with h history frames
    # and window h, step k predicts from frames [k, k+h) and actions [k, k+h)
    cfg = small_config(history=2)
    w = cfg.random_weights(8)
    m = O.LewmModel(cfg, w)
    rng = np.random.default_rng(4)
    B, S, T, h = 1, 3, 4, 2
    emb = rng.standard_normal((B, h, cfg.embed_dim)).astype(np.float32)
    goal = rng.standard_normal((B, cfg.embed_dim)).astype(np.float32)
    cand = rng.uniform(-1, 1, (B, S, T, 2)).astype(np.float32)
    scores, last = m.scores(emb, goal, cand, with_last=True)
    act = m.action_embed(cand.reshape(-1, 2)).reshape(S, T, -1)
    frames = [np.repeat(emb[:, j], S, 0) for j in range(h)]
    for step in range(T - h + 1):
        win = np.stack(frames[step:step + h], 1)
        frames.append(m.predict_last(win, act[:, step:step + h]))
    np.testing.assert_allclose(last[0], frames[-1], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(scores[0], ((frames[-1] - goal[0]) ** 2).sum(-1), rtol=1e-5)
