"""Trained weights from safetensors files into the weight blobs (host only).

The expected VarBuilder paths are restated here from the reference's model
constructors: SkyJepaModel::new (src/models/skyjepa/model.rs:22-39),
TemporalBlock (tcn.rs:54-85), candle's GRU names, SkyJepaProber::new
(prober.rs:54-80), ActionEmbedder / Mlp / ConditionalBlock / Transformer /
Predictor (src/models/lewm/modules.rs:90-372), HfVitEncoder (vit.rs:30-45),
VectorMlpEncoder (src/models/world_model/model.rs:215-250).  Files are
written with the safetensors package, independently of the loader."""
import numpy as np
import pytest

import lewm_b200 as L

st_numpy = pytest.importorskip("safetensors.numpy")


def _tcn_names(cfg, prefix):
    out, cin = [], cfg.input_dim
    for lvl in range(cfg.levels):
        o, k = cfg.channels[lvl], cfg.kernel_size
        b = f"{prefix}.blocks.{lvl}"
        out += [(b + ".conv1.weight", (o, cin, k)), (b + ".conv1.bias", (o,)), (b + ".conv2.weight", (o, o, k)),
                (b + ".conv2.bias", (o,))]
        if cin != o:
            out += [(b + ".residual.weight", (o, cin, 1)), (b + ".residual.bias", (o,))]
        cin = o
    return out


def skyjepa_names(cfg):
    """(latent names, prober names) in blob order."""
    H = cfg.latent_dim
    so = cfg.state_encoder.channels[cfg.state_encoder.levels - 1]
    E = cfg.action_encoder.channels[cfg.action_encoder.levels - 1]
    latent = _tcn_names(cfg.state_encoder, "state_encoder")
    latent += [("state_projection.weight", (H, so)), ("state_projection.bias", (H,))]
    latent += _tcn_names(cfg.action_encoder, "action_encoder")
    latent += [("predictor.weight_ih_l0", (3 * H, E)), ("predictor.weight_hh_l0", (3 * H, H)),
               ("predictor.bias_ih_l0", (3 * H,)), ("predictor.bias_hh_l0", (3 * H,))]
    hid = cfg.prober_hidden_dim
    prober = [("input.weight", (hid, H)), ("input.bias", (hid,))]
    for i in range(cfg.prober_hidden_layers - 1):
        prober += [(f"hidden.{i}.weight", (hid, hid)), (f"hidden.{i}.bias", (hid,))]
    prober += [("output.weight", (15, hid)), ("output.bias", (15,))]
    return latent, prober


def _lin(name, o, i, bias=True):
    return [(name + ".weight", (o, i))] + ([(name + ".bias", (o,))] if bias else [])


def _norm(name, kind, d):
    if kind == L.NORM_KINDS["batch"]:
        return [(name + s, (d,)) for s in (".weight", ".bias", ".running_mean", ".running_var")]
    if kind == L.NORM_KINDS["layer"]:
        return [(name + ".weight", (d,)), (name + ".bias", (d,))]
    return []


def _mlp(name, i, h, o, kind):
    return _lin(name + ".net.0", h, i) + _norm(name + ".net.1", kind, h) + _lin(name + ".net.3", o, h)


def lewm_names(c, naming):
    D, hid, inner = c.embed_dim, c.pred_hidden_dim, c.heads * c.dim_head
    out = [("action_encoder.patch_embed.weight", (c.smoothed_dim, c.action_dim, 1)),
           ("action_encoder.patch_embed.bias", (c.smoothed_dim,))]
    out += _lin("action_encoder.embed.0", c.action_mlp_scale * D, c.smoothed_dim)
    out += _lin("action_encoder.embed.2", D, c.action_mlp_scale * D)
    out += [("predictor.pos_embedding", (1, c.num_frames, D))]
    t = "predictor.transformer"
    if hid != D:
        out += _lin(t + ".input_proj", hid, D) + _lin(t + ".cond_proj", hid, D)
    for i in range(c.depth):
        p = f"{t}.layers.{i}"
        out += _norm(p + ".attn.norm", 1, hid) + _lin(p + ".attn.to_qkv", 3 * inner, hid, bias=False)
        out += _lin(p + ".attn.to_out.0", hid, inner) + _norm(p + ".mlp.net.0", 1, hid)
        out += _lin(p + ".mlp.net.1", c.mlp_dim, hid) + _lin(p + ".mlp.net.4", hid, c.mlp_dim)
        out += _lin(p + ".adaLN_modulation.1", 6 * hid, hid)
    out += _norm(t + ".norm", 1, hid)
    if hid != D:
        out += _lin(t + ".output_proj", D, hid)
    out += _mlp("pred_proj", D, c.pred_proj_hidden, D, c.pred_proj_norm)
    if c.encoder == 0:  # vector MLP (WorldModel only)
        p = "observation_encoder.vector_mlp"
        for j in range(c.obs_depth):
            i = c.obs_dim if j == 0 else c.obs_hidden_dim
            o = D if j + 1 == c.obs_depth else c.obs_hidden_dim
            out += _lin(f"{p}.layers.{j}", o, i)
            if j + 1 < c.obs_depth and c.obs_norm != L.NORM_KINDS["none"]:
                out += _norm(f"{p}.norms.{j}", 1, c.obs_hidden_dim)
    else:
        e = "encoder" if naming == "lewm" else "observation_encoder.encoder"
        vh, p = c.vit_hidden, c.patch_size
        n = (c.image_size // p) ** 2
        out += [(e + ".embeddings.cls_token", (1, 1, vh)), (e + ".embeddings.position_embeddings", (1, n + 1, vh)),
                (e + ".embeddings.patch_embeddings.projection.weight", (vh, c.channels, p, p)),
                (e + ".embeddings.patch_embeddings.projection.bias", (vh,))]
        for i in range(c.vit_layers):
            q = f"{e}.encoder.layer.{i}"
            out += _norm(q + ".layernorm_before", 1, vh)
            for m in ("query", "key", "value"):
                out += _lin(f"{q}.attention.attention.{m}", vh, vh, bias=bool(c.qkv_bias))
            out += _lin(q + ".attention.output.dense", vh, vh) + _norm(q + ".layernorm_after", 1, vh)
            out += _lin(q + ".intermediate.dense", c.vit_mlp, vh) + _lin(q + ".output.dense", vh, c.vit_mlp)
        out += _norm(e + ".layernorm", 1, vh)
        out += _mlp("projector" if naming == "lewm" else "observation_encoder.projector", vh, c.projector_hidden, D,
                    c.projector_norm)
    return out


def _split(blob, names, start=0):
    out, off = {}, start
    for name, shape in names:
        n = int(np.prod(shape))
        out[name] = blob[off:off + n].reshape(shape).copy()
        off += n
    return out, off


def _sky_files(tmp_path, cfg, blob, dtype=np.float32):
    latent, prober = skyjepa_names(cfg)
    lt, off = _split(blob, latent)
    pt, end = _split(blob, prober, off)
    assert end == blob.size
    lp, pp = tmp_path / "latent.safetensors", tmp_path / "prober.safetensors"
    st_numpy.save_file({k: v.astype(dtype) for k, v in lt.items()}, str(lp))
    st_numpy.save_file({k: v.astype(dtype) for k, v in pt.items()}, str(pp))
    return lp, pp, lt, pt


@pytest.mark.parametrize("which", ["paper", "wide"])
def test_skyjepa_names_follow_the_reference(which):
    cfg = getattr(L.SkyJepaConfig, which)()
    latent, prober = skyjepa_names(cfg)
    got = cfg.tensors()
    assert [(t.name, t.shape) for t in got] == latent + prober
    assert [t.file for t in got] == [0] * len(latent) + [1] * len(prober)
    assert sum(t.numel for t in got) == cfg.weight_count()


@pytest.mark.parametrize("which,naming", [("image", "lewm"), ("image", "world_model"), ("vector", "world_model")])
def test_lewm_names_follow_the_reference(which, naming):
    cfg = getattr(L.LewmConfig, which)()
    got = cfg.tensors(naming)
    assert [(t.name, t.shape) for t in got] == lewm_names(cfg, naming)
    assert sum(t.numel for t in got) == cfg.weight_count()
    offs = np.cumsum([0] + [t.numel for t in got])[:-1]
    assert [t.offset for t in got] == offs.tolist()


def test_skyjepa_round_trip_f32(tmp_path):
    cfg = L.SkyJepaConfig.wide()
    blob = cfg.random_weights(3)
    lp, pp, _, _ = _sky_files(tmp_path, cfg, blob)
    assert np.array_equal(cfg.weights_from_safetensors(str(lp), str(pp)), blob)


@pytest.mark.parametrize("dtype", [np.float16, np.float64])
def test_skyjepa_converts_float_widths(tmp_path, dtype):
    cfg = L.SkyJepaConfig.paper()
    blob = cfg.random_weights(4)
    lp, pp, _, _ = _sky_files(tmp_path, cfg, blob, dtype)
    assert np.array_equal(cfg.weights_from_safetensors(str(lp), str(pp)), blob.astype(dtype).astype(np.float32))


def test_bf16_checkpoint(tmp_path):
    torch = pytest.importorskip("torch")
    st_torch = pytest.importorskip("safetensors.torch")
    cfg = L.SkyJepaConfig.paper()
    blob = cfg.random_weights(5)
    latent, prober = skyjepa_names(cfg)
    lt, off = _split(blob, latent)
    pt, _ = _split(blob, prober, off)
    lp, pp = tmp_path / "l.safetensors", tmp_path / "p.safetensors"
    st_torch.save_file({k: torch.from_numpy(v).to(torch.bfloat16) for k, v in lt.items()}, str(lp))
    st_torch.save_file({k: torch.from_numpy(v).to(torch.bfloat16) for k, v in pt.items()}, str(pp))
    want = torch.from_numpy(blob).to(torch.bfloat16).float().numpy()
    assert np.array_equal(cfg.weights_from_safetensors(str(lp), str(pp)), want)


def test_extra_tensors_are_ignored_and_missing_ones_named(tmp_path):
    cfg = L.SkyJepaConfig.paper()
    blob = cfg.random_weights(6)
    _, _, lt, pt = _sky_files(tmp_path, cfg, blob)
    lt["optimizer.step"] = np.zeros(3, np.float32)
    extra = tmp_path / "extra.safetensors"
    st_numpy.save_file(lt, str(extra), metadata={"format": "pt"})
    pp = tmp_path / "prober.safetensors"
    assert np.array_equal(cfg.weights_from_safetensors(str(extra), str(pp)), blob)
    del lt["predictor.weight_hh_l0"]
    st_numpy.save_file(lt, str(extra))
    with pytest.raises(L.LwmError, match=r"cannot find tensor predictor\.weight_hh_l0$"):
        cfg.weights_from_safetensors(str(extra), str(pp))


def test_shape_mismatch_and_bad_files(tmp_path):
    cfg = L.SkyJepaConfig.paper()
    blob = cfg.random_weights(7)
    lp, pp, lt, pt = _sky_files(tmp_path, cfg, blob)
    pt["output.weight"] = pt["output.weight"][:, :-1].copy()
    bad = tmp_path / "bad.safetensors"
    st_numpy.save_file(pt, str(bad))
    h = cfg.prober_hidden_dim
    with pytest.raises(L.LwmError, match=rf"shape mismatch for output\.weight, expected \[15, {h}\], got \[15, {h - 1}\]"):
        cfg.weights_from_safetensors(str(lp), str(bad))
    with pytest.raises(L.LwmError, match="cannot open"):
        cfg.weights_from_safetensors(str(tmp_path / "absent.safetensors"), str(pp))
    trunc = tmp_path / "trunc.safetensors"
    trunc.write_bytes(lp.read_bytes()[:100])
    with pytest.raises(L.LwmError, match="exceeds the file"):
        cfg.weights_from_safetensors(str(trunc), str(pp))
    garbage = tmp_path / "garbage.safetensors"
    garbage.write_bytes((16).to_bytes(8, "little") + b"{not json at all" + b"\0" * 8)
    with pytest.raises(L.LwmError, match="invalid safetensors header"):
        cfg.weights_from_safetensors(str(garbage), str(pp))
    ints = tmp_path / "ints.safetensors"
    st_numpy.save_file({k: (v.astype(np.int32) if k == "input.bias" else v) for k, v in pt.items()}, str(ints))
    with pytest.raises(L.LwmError, match="unsupported dtype I32 for tensor input.bias"):
        cfg.weights_from_safetensors(str(lp), str(ints))


@pytest.mark.parametrize("which,naming", [("image", "lewm"), ("vector", "world_model")])
def test_lewm_round_trip(tmp_path, which, naming):
    cfg = getattr(L.LewmConfig, which)()
    blob = cfg.random_weights(8)
    tensors, end = _split(blob, lewm_names(cfg, naming))
    assert end == blob.size
    path = tmp_path / "w.safetensors"
    st_numpy.save_file(tensors, str(path))
    assert np.array_equal(cfg.weights_from_safetensors(str(path), naming), blob)


def test_lewm_naming_needs_a_vit(tmp_path):
    cfg = L.LewmConfig.vector()
    assert cfg.tensors("lewm") == []
    with pytest.raises(L.LwmError, match="LeWm checkpoints hold a ViT observation encoder"):
        cfg.weights_from_safetensors(str(tmp_path / "x.safetensors"), "lewm")
