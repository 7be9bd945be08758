"""SkyJEPA checkpoint packages: `checkpoint.json` plus content-addressed
`objects/<sha256>.safetensors` (SkyJepaCheckpoint::load,
src/models/skyjepa/checkpoint.rs:65-215).

`load_skyjepa_package(root)` checks the package as the reference loader does
— format version 2, the contract (model, dataset, normalisation, prober) and
its fingerprint, the sha256 of every weights object — and returns what the
learned scorer and the controller session take: the model configuration, the
weight blob (lwm_skyjepa_weights_from_safetensors on the latent and prober
objects) and the normalisation.

The contract fingerprint is the sha256 of the contract serialised compactly
by serde_json.  The numbers are re-emitted with the exact text they have in
`checkpoint.json` (serde writes the same digits pretty or compact), so the
fingerprint of a package the reference published verifies here.
"""
from __future__ import annotations

import hashlib
import json
import os
from dataclasses import dataclass

import numpy as np

from . import LwmError, SkyJepaConfig

CHECKPOINT_VERSION = 2
STATE_DIM, ACTION_DIM = 18, 4
MODEL_RATE_HZ = 20
ACTION_SPACES = {"body_rates_throttle": 0, "rotor_forces": 1}


class CheckpointError(LwmError):
    def __init__(self, message: str):
        super().__init__(1, message)


class _Number(str):
    """A JSON number kept as the text it was written with."""


def _compact(value) -> str:
    """serde_json::to_vec of a value parsed from JSON: no whitespace, object
    keys in file order, numbers as written."""
    if isinstance(value, dict):
        return "{" + ",".join(json.dumps(k, ensure_ascii=False) + ":" + _compact(v) for k, v in value.items()) + "}"
    if isinstance(value, list):
        return "[" + ",".join(_compact(v) for v in value) + "]"
    if isinstance(value, _Number):
        return str(value)
    if value is True:
        return "true"
    if value is False:
        return "false"
    if value is None:
        return "null"
    return json.dumps(value, ensure_ascii=False)


def _sha256_file(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 16), b""):
            h.update(chunk)
    return h.hexdigest()


def contract_sha256(contract_json_text: str) -> str:
    """Fingerprint of a contract given as JSON text (json_sha256, checkpoint.rs:191-193)."""
    parsed = json.loads(contract_json_text, parse_float=_Number, parse_int=_Number)
    return hashlib.sha256(_compact(parsed).encode()).hexdigest()


def _ensure(cond: bool, message: str) -> None:
    if not cond:
        raise CheckpointError(message)


def _int(v) -> int:
    return int(str(v))


def _float(v) -> float:
    return float(str(v))


def _object_path(root: str, digest: str) -> str:
    return os.path.join(root, "objects", f"{digest}.safetensors")


def _verify_object(root: str, digest) -> str:
    _ensure(isinstance(digest, str) and len(digest) == 64 and all(c in "0123456789abcdefABCDEF" for c in digest),
            "invalid checkpoint object hash")
    path = _object_path(root, digest)
    _ensure(os.path.exists(path) and _sha256_file(path) == digest, f"checkpoint weights fingerprint mismatch: {digest}")
    return path


def _tcn(cfg_tcn, src: dict, name: str) -> None:
    chans = [_int(c) for c in src["channels"]]
    _ensure(_int(src["input_dim"]) > 0, f"{name}.input_dim must be greater than zero")
    _ensure(len(chans) > 0, f"{name}.channels must not be empty")
    _ensure(all(c > 0 for c in chans), f"{name}.channels must all be greater than zero")
    _ensure(_int(src["kernel_size"]) > 0, f"{name}.kernel_size must be greater than zero")
    _ensure(len(chans) <= len(cfg_tcn.channels), f"{name} has more levels than this library supports")
    cfg_tcn.input_dim = _int(src["input_dim"])
    cfg_tcn.levels = len(chans)
    cfg_tcn.kernel_size = _int(src["kernel_size"])
    for i, c in enumerate(chans):
        cfg_tcn.channels[i] = c


@dataclass
class SkyJepaPackage:
    root: str
    config: SkyJepaConfig
    weights: np.ndarray
    state_mean: np.ndarray
    state_std: np.ndarray
    action_mean: np.ndarray
    action_std: np.ndarray
    dataset: dict
    provenance: object
    fingerprint: str

    @property
    def dt(self) -> float:
        """Control period of the session: 1 / model_rate_hz (session.rs:204)."""
        return 1.0 / _int(self.dataset["model_rate_hz"])


def load_skyjepa_package(root: str) -> SkyJepaPackage:
    path = os.path.join(root, "checkpoint.json")
    try:
        with open(path, "r", encoding="utf-8") as f:
            text = f.read()
        data = json.loads(text, parse_float=_Number, parse_int=_Number)
    except (OSError, ValueError) as exc:
        raise CheckpointError("SkyJEPA requires a versioned checkpoint package, not loose safetensors") from exc
    _ensure(_int(data.get("format_version", -1)) == CHECKPOINT_VERSION, "unsupported SkyJEPA checkpoint version")
    contract = data["contract"]
    model, dataset, norm, prober = contract["model"], contract["dataset"], contract["normalization"], contract.get("prober")
    # ModelContract::validate (checkpoint.rs:32-60)
    _ensure(_int(model["state_dim"]) == STATE_DIM and _int(model["action_dim"]) == ACTION_DIM,
            "checkpoint requires state18/action4")
    _ensure(_int(model["history_steps"]) == _int(dataset["history_steps"])
            and _int(model["rollout_steps"]) == _int(dataset["rollout_steps"]),
            "checkpoint model/dataset sequence dimensions disagree")
    _ensure(bool(dataset["normalize_states"]) and bool(dataset["normalize_actions"]),
            "checkpoint requires normalized state/action model inputs")
    _ensure(_int(dataset["model_rate_hz"]) == MODEL_RATE_HZ,
            f"SkyJEPA requires the canonical {MODEL_RATE_HZ} Hz model rate")
    for name, dim in (("state", STATE_DIM), ("action", ACTION_DIM)):
        mean = [_float(v) for v in norm[name]["mean"]]
        std = [_float(v) for v in norm[name]["std"]]
        _ensure(len(mean) == dim and len(std) == dim,
                f"fixed {name} normalization has mean/std dimensions {len(mean)}/{len(std)}; expected {dim}")
        _ensure(all(np.isfinite(mean)), f"fixed {name} normalization mean contains non-finite values")
        _ensure(all(np.isfinite(v) and v > 0 for v in std), f"fixed {name} normalization std must be finite and positive")
    if prober is not None:
        _ensure(_int(prober["latent_dim"]) == _int(model["latent_dim"])
                and prober["kinematics"]["action_space"] == dataset["action_space"],
                "checkpoint prober/model/action-space mismatch")
    _ensure(hashlib.sha256(_compact(contract).encode()).hexdigest() == data.get("contract_sha256"),
            "checkpoint contract fingerprint mismatch")
    _ensure((prober is None) == (data.get("prober_sha256") is None), "checkpoint prober weights/configuration mismatch")
    latent = _verify_object(root, data.get("latent_sha256"))
    _ensure(prober is not None, "control requires a trained prober")
    prober_path = _verify_object(root, data["prober_sha256"])
    cfg = SkyJepaConfig()
    cfg.state_dim, cfg.action_dim = STATE_DIM, ACTION_DIM
    cfg.history_steps, cfg.rollout_steps = _int(model["history_steps"]), _int(model["rollout_steps"])
    cfg.latent_dim = _int(model["latent_dim"])
    _tcn(cfg.state_encoder, model["state_encoder"], "state_encoder")
    _tcn(cfg.action_encoder, model["action_encoder"], "action_encoder")
    cfg.prober_hidden_dim = _int(prober["hidden_dim"])
    cfg.prober_hidden_layers = _int(prober["hidden_layers"])
    kin = prober["kinematics"]
    cfg.kinematics.mass, cfg.kinematics.gravity = _float(kin["mass"]), _float(kin["gravity"])
    cfg.kinematics.hover_throttle = _float(kin["hover_throttle"])
    _ensure(kin["action_space"] in ACTION_SPACES, f"unknown action space {kin['action_space']!r}")
    cfg.kinematics.action_space = ACTION_SPACES[kin["action_space"]]
    weights = cfg.weights_from_safetensors(latent, prober_path)
    f32 = lambda xs: np.array([_float(v) for v in xs], np.float32)
    fingerprint = hashlib.sha256(_compact(data).encode()).hexdigest()
    return SkyJepaPackage(root, cfg, weights, f32(norm["state"]["mean"]), f32(norm["state"]["std"]),
                          f32(norm["action"]["mean"]), f32(norm["action"]["std"]), dataset,
                          data.get("provenance"), fingerprint)
