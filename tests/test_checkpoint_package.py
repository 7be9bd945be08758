"""SkyJEPA checkpoint packages (checkpoint.json + objects/<sha256>.safetensors;
SkyJepaCheckpoint::load, src/models/skyjepa/checkpoint.rs:65-215), host only.

The package is written here the way SkyJepaCheckpoint::publish writes it
(pretty JSON manifest, contract fingerprint = sha256 of the compact contract,
weights stored under their own sha256), with numbers whose text Python and
serde_json write alike."""
import hashlib
import json
import os

import numpy as np
import pytest

import lewm_b200 as L
from lewm_b200.checkpoint import CheckpointError, load_skyjepa_package

st_numpy = pytest.importorskip("safetensors.numpy")
from test_checkpoint import _split, skyjepa_names  # noqa: E402


def _contract(cfg):
    tcn = lambda t: {"input_dim": t.input_dim, "channels": [t.channels[i] for i in range(t.levels)],
                     "kernel_size": t.kernel_size}
    return {
        "model": {"state_dim": 18, "action_dim": 4, "history_steps": cfg.history_steps,
                  "rollout_steps": cfg.rollout_steps, "latent_dim": cfg.latent_dim,
                  "state_encoder": tcn(cfg.state_encoder), "action_encoder": tcn(cfg.action_encoder)},
        "dataset": {"batch_size": 64, "history_steps": cfg.history_steps, "rollout_steps": cfg.rollout_steps,
                    "model_rate_hz": 20, "normalize_states": True, "normalize_actions": True,
                    "action_space": "rotor_forces", "split_by": "episodes"},
        "normalization": {"state": {"mean": [0.25] * 18, "std": [2.0] * 18},
                          "action": {"mean": [3.0] * 4, "std": [0.5] * 4}},
        "prober": {"latent_dim": cfg.latent_dim, "hidden_dim": cfg.prober_hidden_dim,
                   "hidden_layers": cfg.prober_hidden_layers,
                   "kinematics": {"mass": 1.3, "gravity": 9.81, "hover_throttle": 0.2, "action_space": "rotor_forces"}},
    }


def _publish(root, cfg, blob, contract=None, version=2):
    os.makedirs(os.path.join(root, "objects"), exist_ok=True)
    latent, prober = skyjepa_names(cfg)
    lt, off = _split(blob, latent)
    pt, _ = _split(blob, prober, off)
    digests = []
    for tensors in (lt, pt):
        tmp = os.path.join(root, "tmp.safetensors")
        st_numpy.save_file(tensors, tmp)
        digest = hashlib.sha256(open(tmp, "rb").read()).hexdigest()
        os.replace(tmp, os.path.join(root, "objects", f"{digest}.safetensors"))
        digests.append(digest)
    contract = contract or _contract(cfg)
    manifest = {"format_version": version, "contract": contract,
                "contract_sha256": hashlib.sha256(json.dumps(contract, separators=(",", ":")).encode()).hexdigest(),
                "latent_sha256": digests[0], "prober_sha256": digests[1], "provenance": {"source": "test"}}
    with open(os.path.join(root, "checkpoint.json"), "w") as f:
        json.dump(manifest, f, indent=2)
    return manifest


def test_load_package(tmp_path):
    cfg = L.SkyJepaConfig.paper()
    cfg.kinematics.action_space = 1
    blob = cfg.random_weights(21)
    _publish(str(tmp_path), cfg, blob)
    pkg = load_skyjepa_package(str(tmp_path))
    assert np.array_equal(pkg.weights, blob)
    assert pkg.config.latent_dim == 24 and pkg.config.prober_hidden_dim == 32
    assert [pkg.config.action_encoder.channels[i] for i in range(3)] == [4, 4, 8]
    assert pkg.config.kinematics.action_space == 1 and pkg.config.kinematics.mass == pytest.approx(1.3)
    assert pkg.dt == pytest.approx(0.05)
    assert pkg.state_std.tolist() == [2.0] * 18 and pkg.action_mean.tolist() == [3.0] * 4
    assert pkg.config.weight_count() == blob.size


def test_contract_fingerprint_uses_the_written_number_text(tmp_path):
    # a manifest written with other whitespace still verifies; a changed digit does not
    cfg = L.SkyJepaConfig.paper()
    man = _publish(str(tmp_path), cfg, cfg.random_weights(22))
    path = os.path.join(str(tmp_path), "checkpoint.json")
    with open(path, "w") as f:
        json.dump(man, f, indent=4)
    load_skyjepa_package(str(tmp_path))
    text = open(path).read().replace('"hover_throttle": 0.2', '"hover_throttle": 0.20', 1)
    open(path, "w").write(text)
    with pytest.raises(CheckpointError, match="checkpoint contract fingerprint mismatch"):
        load_skyjepa_package(str(tmp_path))


def test_package_errors(tmp_path):
    cfg = L.SkyJepaConfig.paper()
    root = str(tmp_path / "a")
    with pytest.raises(CheckpointError, match="not loose safetensors"):
        load_skyjepa_package(root)
    man = _publish(root, cfg, cfg.random_weights(23), version=1)
    with pytest.raises(CheckpointError, match="unsupported SkyJEPA checkpoint version"):
        load_skyjepa_package(root)
    man = _publish(root, cfg, cfg.random_weights(23))
    obj = os.path.join(root, "objects", man["latent_sha256"] + ".safetensors")
    data = bytearray(open(obj, "rb").read())
    data[-1] ^= 1
    open(obj, "wb").write(bytes(data))
    with pytest.raises(CheckpointError, match="checkpoint weights fingerprint mismatch: " + man["latent_sha256"]):
        load_skyjepa_package(root)
    c = _contract(cfg)
    c["dataset"]["model_rate_hz"] = 30
    _publish(str(tmp_path / "b"), cfg, cfg.random_weights(24), contract=c)
    with pytest.raises(CheckpointError, match="canonical 20 Hz model rate"):
        load_skyjepa_package(str(tmp_path / "b"))
    c = _contract(cfg)
    c["normalization"]["state"]["std"][3] = 0.0
    _publish(str(tmp_path / "c"), cfg, cfg.random_weights(25), contract=c)
    with pytest.raises(CheckpointError, match="state normalization std must be finite and positive"):
        load_skyjepa_package(str(tmp_path / "c"))
