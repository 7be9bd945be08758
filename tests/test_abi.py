"""The C ABI without a GPU: the library loads, exports every symbol the header
declares, and its host-side logic (config defaults, validation messages,
task inputs, weight layout) agrees with the reference and the oracle."""
import ctypes as C
import os
import re

import numpy as np
import pytest

import lewm_b200 as L
import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared(header: str, prefix: str):
    text = open(header).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(rf"\b({prefix}\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    names = _declared(os.path.join(ROOT, "include", "lewm_b200.h"), "lwm_")
    assert len(names) >= 40
    lib = C.CDLL(L.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_oracle_exports_every_declared_symbol():
    names = _declared(os.path.join(ROOT, "oracle", "lewm_oracle.h"), "orc_")
    lib = C.CDLL(O.LIB_PATH)
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_abi_version_and_version_string():
    assert L.lib.lwm_abi_version() == 1
    assert "sm_100a" in L.version()


def test_config_defaults_mirror_reference_constructors():
    # MppiConfig::new / CemConfig::new / IcemConfig::new (src/planner.rs:122-137, 193-208, 275-295)
    m = L.MppiConfig(15, 512, 4)._c()
    assert (m.iterations, m.noise_std, m.temperature, m.has_seed, m.deadline_ns) == (1, 1.0, 1.0, 0, -1)
    assert list(m.bounds_low[:4]) == [-1.0] * 4 and list(m.bounds_high[:4]) == [1.0] * 4
    c = L.CemConfig(5, 300, 30, 2)._c()
    assert (c.iterations, c.init_std, c.elites) == (4, 1.0, 30) and abs(c.min_std - 1e-3) < 1e-9
    i = L.IcemConfig(5, 300, 30, 2)._c()
    assert (i.keep_elites, i.iterations, i.noise_beta, i.return_mean) == (30, 4, 2.0, 1)
    assert abs(i.alpha - 0.1) < 1e-7


def _create_error(kind, cfg):
    fn = {"mppi": L.lib.lwm_mppi_create, "cem": L.lib.lwm_cem_create, "icem": L.lib.lwm_icem_create}[kind]
    out = C.c_void_p()
    status = fn(None, C.byref(cfg._c()), C.byref(out))
    return status, L.lib.lwm_last_error().decode()


@pytest.mark.parametrize("kind,cfg,message", [
    ("mppi", L.MppiConfig(0, 4, 2), "MPPI horizon must be greater than zero"),
    ("mppi", L.MppiConfig(3, 0, 2), "MPPI samples must be greater than zero"),
    ("mppi", L.MppiConfig(3, 4, 2, iterations=0), "MPPI iterations must be greater than zero"),
    ("mppi", L.MppiConfig(3, 4, 2, noise_std=0.0), "MPPI noise_std must be finite and greater than zero"),
    ("mppi", L.MppiConfig(3, 4, 2, noise_std_per_action=[0.1, -1.0]),
     "MPPI per-action noise values must be finite and greater than zero"),
    ("mppi", L.MppiConfig(3, 4, 2, temperature=float("nan")), "MPPI temperature must be finite and greater than zero"),
    ("mppi", L.MppiConfig(3, 4, 2, action_bounds=L.ActionBounds([1.0, 0.0], [0.0, 1.0])),
     "action bound 0 has low 1 greater than high 0"),
    ("mppi", L.MppiConfig(3, 4, 2, action_bounds=L.ActionBounds([0.0, float("inf")], [1.0, 1.0])),
     "action bound 1 is not finite"),
    ("mppi", L.MppiConfig(3, 4, 2, deadline_action=[0.0, 1.5]), "MPPI deadline_action[1]=1.5 is outside [-1, 1]"),
    ("cem", L.CemConfig(3, 4, 1, 2), "CEM elites must be at least two"),
    ("cem", L.CemConfig(3, 4, 5, 2), "CEM elites 5 cannot exceed samples 4"),
    ("cem", L.CemConfig(3, 4, 2, 2, min_std=-1.0), "CEM min_std must be finite and non-negative"),
    ("cem", L.CemConfig(3, 4, 2, 2, init_std=0.0), "CEM init_std must be finite and greater than zero"),
    ("icem", L.IcemConfig(3, 4, 5, 2), "iCEM elites 5 cannot exceed samples 4 on the first iteration"),
    ("icem", L.IcemConfig(3, 4, 2, 2, keep_elites=3), "iCEM keep_elites 3 cannot exceed elites 2"),
    ("icem", L.IcemConfig(3, 4, 2, 2, alpha=1.5), "iCEM alpha must be finite and in [0, 1]"),
    ("icem", L.IcemConfig(3, 4, 2, 2, noise_beta=-1.0), "iCEM noise_beta must be finite and non-negative"),
])
def test_validation_messages_match_reference(kind, cfg, message):
    # src/planner.rs:85-103, 139-175, 210-253, 296-345, 1060-1089
    status, msg = _create_error(kind, cfg)
    assert status == 1
    assert msg == message


def test_valid_config_then_requires_context():
    status, msg = _create_error("mppi", L.MppiConfig(3, 4, 2))
    assert status == 1 and msg == "null argument"


def test_image_control_step_rejects_null_handles():
    # lwm_lewm_plan_nv12_device checks its arguments before any device work
    cfg = L.ImagePreprocess.imagenet_224()
    r = L._PlanDeviceResult()
    status = L.lib.lwm_lewm_plan_nv12_device(None, None, None, None, 1, 1, 224, 224, 0, C.byref(cfg), None,
                                              C.byref(r))
    assert status == 1 and L.lib.lwm_last_error().decode() == "null argument"


def test_unsupported_sizes_are_rejected_loudly():
    status, msg = _create_error("mppi", L.MppiConfig(65, 4, 2))
    assert status == 6 and "horizon 65" in msg
    status, msg = _create_error("mppi", L.MppiConfig(3, 4, 17))
    assert status == 6


@pytest.mark.parametrize("kind", ["hover", "circle", "figure-eight"])
def test_reference_horizon_matches_oracle(kind):
    ours = L.reference_horizon(kind, 1.3, 0.05, 15, 2.0, 8.0)
    k = L.REFERENCE_KINDS[kind]
    ref = np.stack([O.reference_state(k, np.float32(1.3) + np.float32(i) * np.float32(0.05), 2.0, 8.0)
                    for i in range(1, 16)])
    assert np.abs(ours - ref).max() < 1e-6


def test_geometric_prior_matches_oracle():
    rng = np.random.default_rng(0)
    refs = L.reference_horizon("figure-eight", 0.7, 0.05, 15, 2.0, 8.0)
    cur = refs[0].copy()
    cur[0:6] += rng.normal(0, 0.1, 6).astype(np.float32)
    ours = L.geometric_prior(cur, refs, 0.05)
    ref = O.geometric_prior(cur, refs, 0.05)
    assert np.abs(ours - ref).max() < 1e-5


def test_plant_step_matches_oracle():
    d = L.Domain.sample(918)
    rng = np.random.default_rng(1)
    x1 = L.hover_state(); x1[3:6] = [0.3, -0.2, 0.1]; x1[15:18] = [0.4, -0.2, 0.3]
    x2 = x1.copy()
    m1 = np.full(4, d.hover_force(), np.float32); m2 = m1.copy()
    for _ in range(200):
        cmd = (d.hover_force() + rng.normal(0, 0.3, 4)).astype(np.float32)
        L.plant_step(d, x1, m1, cmd, 0.005)
        O.plant_step(d, x2, m2, cmd, 0.005)
    assert np.abs(x1 - x2).max() < 1e-5


def test_domain_sample_matches_reference_ranges_and_is_deterministic():
    a, b = L.Domain.sample(918), L.Domain.sample(918)
    assert bytes(a) == bytes(b)
    assert 0.65 <= a.mass <= 1.95


@pytest.mark.parametrize("make", [L.SkyJepaConfig.paper, L.SkyJepaConfig.wide])
def test_weight_layout_count_matches_oracle_layout(make):
    cfg = make()
    assert cfg.weight_count() == O.skyjepa_weight_count(cfg)
    w = cfg.random_weights(7)
    assert w.size == cfg.weight_count() and np.isfinite(w).all()
    assert np.array_equal(w, cfg.random_weights(7))
    assert not np.array_equal(w, cfg.random_weights(8))


def test_workloads_are_deterministic():
    from lewm_b200 import workloads as W
    a, b = W.skyjepa(3), W.skyjepa(3)
    assert np.array_equal(a.state_history, b.state_history) and np.array_equal(a.weights, b.weights)
    assert a.state_history.shape == (1, 10, 18) and a.reference_states.shape == (1, 15, 18)
