"""ctypes wrapper of the CPU oracle (liblewm_oracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as the
checker, and by bench.py's CPU-baseline / reference leg.  The product library
(le-wm-nv_b200) never imports, links or calls this module.

The library is built by oracle/Makefile (`make -C oracle`).
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblewm_oracle.so")
if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `make -C oracle`")
lib = C.CDLL(LIB_PATH)

F = C.c_float
U32 = C.c_uint32
U64 = C.c_uint64
I32 = C.c_int32
FP = C.POINTER(C.c_float)
UP = C.POINTER(C.c_uint32)
VP = C.c_void_p
SCORE_FN = C.CFUNCTYPE(None, VP, FP, U32, U32, U32, U32, FP)

# ---- ctypes mirrors of the structs of include/lewm_b200.h that the oracle's
# C interface takes (the oracle includes that header for its types).  This
# module defines its own and imports nothing from the product package; a
# product struct instance handed in by a test is copied byte for byte into the
# mirror (_own), the layouts being the same header's.
MAX_ACTION_DIM = 16
TCN_MAX_LEVELS = 8


class _MppiConfig(C.Structure):
    _fields_ = [("horizon", U32), ("samples", U32), ("iterations", U32), ("action_dim", U32),
                ("bounds_low", F * MAX_ACTION_DIM), ("bounds_high", F * MAX_ACTION_DIM), ("noise_std", F),
                ("has_noise_std_per_action", I32), ("noise_std_per_action", F * MAX_ACTION_DIM), ("temperature", F),
                ("deadline_ns", C.c_int64), ("has_deadline_action", I32), ("deadline_action", F * MAX_ACTION_DIM),
                ("has_seed", I32), ("seed", U64)]


class _CemConfig(C.Structure):
    _fields_ = [("horizon", U32), ("samples", U32), ("elites", U32), ("iterations", U32), ("action_dim", U32),
                ("bounds_low", F * MAX_ACTION_DIM), ("bounds_high", F * MAX_ACTION_DIM), ("init_std", F),
                ("min_std", F), ("deadline_ns", C.c_int64), ("has_deadline_action", I32),
                ("deadline_action", F * MAX_ACTION_DIM), ("has_seed", I32), ("seed", U64)]


class _IcemConfig(C.Structure):
    _fields_ = [("horizon", U32), ("samples", U32), ("elites", U32), ("keep_elites", U32), ("iterations", U32),
                ("noise_beta", F), ("alpha", F), ("action_dim", U32), ("bounds_low", F * MAX_ACTION_DIM),
                ("bounds_high", F * MAX_ACTION_DIM), ("init_std", F), ("min_std", F), ("return_mean", I32),
                ("deadline_ns", C.c_int64), ("has_deadline_action", I32), ("deadline_action", F * MAX_ACTION_DIM),
                ("has_seed", I32), ("seed", U64)]


class Domain(C.Structure):
    """SkyJepaDomain (src/skyjepa_sim.rs:28-56)."""
    _fields_ = [("mass", F), ("inertia", F * 3), ("motor_time_constant", F), ("drag", F * 3), ("thrust_scale", F),
                ("torque_scale", F), ("arm_length", F), ("gravity", F), ("max_thrust_weight", F)]

    @staticmethod
    def default() -> "Domain":
        d = Domain()
        lib.orc_domain_default(C.byref(d))
        return d

    def hover_force(self) -> float:
        return float(np.float32(self.mass) * np.float32(self.gravity) / (np.float32(4.0) * np.float32(self.thrust_scale)))


class TrackingCost(C.Structure):
    """SkyJepaTrackingCost (src/models/skyjepa/control.rs:19-37)."""
    _fields_ = [("position", F), ("velocity", F), ("attitude", F), ("angular_velocity", F), ("action", F * 4)]

    @staticmethod
    def paper() -> "TrackingCost":
        c = TrackingCost()
        lib.orc_tracking_cost_paper(C.byref(c))
        return c

    @staticmethod
    def make(position, velocity, attitude, angular_velocity, action) -> "TrackingCost":
        return TrackingCost(position, velocity, attitude, angular_velocity, (F * 4)(*action))


class TcnConfig(C.Structure):
    _fields_ = [("input_dim", U32), ("levels", U32), ("channels", U32 * TCN_MAX_LEVELS), ("kernel_size", U32)]


class KinematicConfig(C.Structure):
    _fields_ = [("mass", C.c_double), ("gravity", C.c_double), ("hover_throttle", C.c_double), ("action_space", I32)]


class SkyJepaConfig(C.Structure):
    """SkyJepaConfig + SkyJepaProberConfig (config.rs:45-55, prober.rs:10-16)."""
    _fields_ = [("state_dim", U32), ("action_dim", U32), ("history_steps", U32), ("rollout_steps", U32),
                ("latent_dim", U32), ("state_encoder", TcnConfig), ("action_encoder", TcnConfig),
                ("prober_hidden_dim", U32), ("prober_hidden_layers", U32), ("kinematics", KinematicConfig)]

    @staticmethod
    def paper() -> "SkyJepaConfig":
        c = SkyJepaConfig()
        lib.orc_skyjepa_config(0, C.byref(c))
        return c

    @staticmethod
    def wide() -> "SkyJepaConfig":
        c = SkyJepaConfig()
        lib.orc_skyjepa_config(1, C.byref(c))
        return c

    def weight_count(self) -> int:
        return int(lib.orc_skyjepa_weight_count(C.byref(self)))

    def random_weights(self, seed: int) -> np.ndarray:
        n = self.weight_count()
        out = np.empty(n, dtype=np.float32)
        if n == 0 or lib.orc_skyjepa_random_weights(C.byref(self), U64(seed), fp(out), C.c_size_t(n)) != 0:
            raise ValueError("invalid SkyJEPA configuration")
        return out


class SessionConfig(C.Structure):
    """SkyJepaSessionConfig + SkyJepaControlConfig (session.rs:40-87, control.rs:72-94)."""
    _fields_ = [("samples", U32), ("horizon", U32), ("planner_seed", U64), ("warm_start", I32),
                ("residual_limit_n", F), ("dynamics", I32), ("trim_multiplier", F), ("dt", F), ("iterations", U32),
                ("temperature", F), ("action_noise", F * 4), ("cost", TrackingCost)]


def skyjepa_weight_count(cfg) -> int:
    return int(lib.orc_skyjepa_weight_count(C.byref(_own(SkyJepaConfig, cfg))))


def _own(cls, obj):
    """obj as this module's mirror `cls` (a product struct of the same header
    layout is copied byte for byte)."""
    if obj is None or isinstance(obj, cls):
        return obj
    if C.sizeof(obj) != C.sizeof(cls):
        raise TypeError(f"{type(obj).__name__} does not have the layout of {cls.__name__}")
    return cls.from_buffer_copy(obj)


class NominalCtx(C.Structure):
    _fields_ = [("initial", FP), ("motors", FP), ("ref_states", FP), ("ref_actions", FP), ("cost", TrackingCost),
                ("dt", F), ("trim_scale", F), ("substeps", U32), ("domain", Domain), ("domains", C.POINTER(Domain))]


class SkyCtx(C.Structure):
    _fields_ = [("model", VP), ("state_mean", FP), ("state_std", FP), ("action_mean", FP), ("action_std", FP),
                ("state_hist", FP), ("action_hist", FP), ("ref_states", FP), ("ref_actions", FP),
                ("cost", TrackingCost), ("dt", F), ("masses", FP)]


def _sig(name, restype, *args):
    f = getattr(lib, name)
    f.restype = restype
    f.argtypes = list(args)


_sig("orc_set_threads", None, C.c_int)
_sig("orc_get_threads", C.c_int)
_sig("orc_philox4x32_10", None, U64, U64, UP)
_sig("orc_normal_at", F, U64, U64)
_sig("orc_normals", None, U64, U64, C.c_size_t, FP)
_sig("orc_sample", None, FP, FP, FP, FP, FP, U32, U32, U32, U32, FP)
_sig("orc_color_noise", None, FP, FP, U32, U32, U32, U32, F)
_sig("orc_inject_carried", None, FP, FP, U32, U32, U32, U32, U32, U32)
_sig("orc_mppi_weighted", None, FP, FP, U32, U32, U32, U32, F, FP)
_sig("orc_lowest_k", None, FP, U32, U32, U32, UP)
_sig("orc_gather", None, FP, UP, U32, U32, U32, U32, U32, FP)
_sig("orc_refit", None, FP, U32, U32, U32, U32, F, FP, FP)
_sig("orc_momentum", None, FP, FP, C.c_size_t, F, FP)
_sig("orc_shift", None, FP, U32, U32, U32, FP)
_sig("orc_plant_step", None, C.POINTER(Domain), FP, FP, FP, F)
_sig("orc_nominal_rollout", None, FP, FP, FP, U32, U32, F, U32, C.POINTER(Domain), FP)
_sig("orc_nominal_rollout_k4", None, FP, FP, FP, U32, U32, F, U32, C.POINTER(Domain), FP)
_sig("orc_tracking_scores", None, FP, FP, FP, FP, C.POINTER(TrackingCost), U32, U32, U32, FP)
_sig("orc_nominal_scores", None, FP, FP, FP, FP, C.POINTER(TrackingCost), F, F, U32, C.POINTER(Domain),
     C.POINTER(Domain), FP, U32, U32, U32, FP, FP)
_sig("orc_skyjepa_new", VP, C.POINTER(SkyJepaConfig), FP, C.c_size_t)
_sig("orc_skyjepa_set_tensor_core_rounding", None, VP)
_sig("orc_skyjepa_free", None, VP)
_sig("orc_skyjepa_weight_count", C.c_size_t, C.POINTER(SkyJepaConfig))
_sig("orc_tcn_forward_last", None, VP, C.c_int, FP, U32, U32, FP)
_sig("orc_initial_latent", None, VP, FP, U32, FP)
_sig("orc_gru_step", None, VP, FP, FP, U32, FP)
_sig("orc_rollout_latents", None, VP, FP, FP, FP, U32, U32, U32, FP)
_sig("orc_prober", None, VP, FP, U32, FP)
_sig("orc_integrate_k3", None, FP, FP, FP, FP, FP, U32, U32, C.POINTER(KinematicConfig), FP)
_sig("orc_integrate_reference", None, FP, FP, FP, FP, FP, U32, U32, C.POINTER(KinematicConfig), FP)
_sig("orc_so3_exp", None, FP, FP)
_sig("orc_skyjepa_scores", None, VP, FP, FP, FP, FP, FP, FP, FP, FP, C.POINTER(TrackingCost), F, FP, U32, U32,
     U32, FP, FP, FP)
_sig("orc_mppi_plan", C.c_int, C.POINTER(_MppiConfig), FP, U32, FP, U64, U64, VP, VP, FP, FP, UP, FP, FP)
_sig("orc_cem_plan", C.c_int, C.POINTER(_CemConfig), U32, FP, U64, U64, VP, VP, FP, FP, UP, FP, UP, FP)
_sig("orc_icem_plan", C.c_int, C.POINTER(_IcemConfig), FP, U32, FP, U64, U64, VP, VP, FP, FP, UP, FP, FP, UP, FP)
_sig("orc_icem_trace", C.c_int, C.POINTER(_IcemConfig), FP, U32, FP, U64, U64, VP, VP, FP, FP, UP, FP, FP)
_sig("orc_reference_state", None, C.c_int, F, F, F, FP)
_sig("orc_domain_default", None, C.POINTER(Domain))
_sig("orc_tracking_cost_paper", None, C.POINTER(TrackingCost))
_sig("orc_skyjepa_config", None, C.c_int, C.POINTER(SkyJepaConfig))
_sig("orc_skyjepa_random_weights", C.c_int, C.POINTER(SkyJepaConfig), U64, FP, C.c_size_t)
_sig("orc_geometric_prior", None, FP, FP, U32, F, C.POINTER(Domain), FP)
_sig("orc_lewm_weight_count", C.c_size_t, C.c_void_p)
_sig("orc_lewm_new", VP, C.c_void_p, FP, C.c_size_t)
_sig("orc_lewm_free", None, VP)
_sig("orc_lewm_action_embed", None, VP, FP, U32, FP)
_sig("orc_lewm_predict_last", None, VP, FP, FP, U32, U32, FP)
_sig("orc_lewm_scores", None, VP, FP, U32, FP, FP, U32, U32, U32, U32, FP, FP)
_sig("orc_lewm_encode_vector", None, VP, FP, U32, FP)
_sig("orc_lewm_encode_pixels", None, VP, FP, U32, FP)
_sig("orc_preprocess_packed", None, C.c_void_p, U32, U32, U32, U32, U32, U32, FP, FP, U32, U32, FP)
_sig("orc_preprocess_nv12", None, C.c_void_p, C.c_void_p, U32, U32, U32, U32, U32, U32, FP, FP, U32, U32, FP)

NOMINAL_FN = C.cast(lib.orc_nominal_score_fn, VP)
SKYJEPA_FN = C.cast(lib.orc_skyjepa_score_fn, VP)


def f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def fp(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"], (a.dtype, a.flags)
    return a.ctypes.data_as(FP)


def up(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.dtype == np.uint32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(UP)


def set_threads(n: int) -> None:
    lib.orc_set_threads(n)


def normals(seed: int, offset: int, count: int) -> np.ndarray:
    out = np.empty(count, np.float32)
    lib.orc_normals(seed, offset, count, fp(out))
    return out


def philox(counter: int, key: int) -> np.ndarray:
    out = np.empty(4, np.uint32)
    lib.orc_philox4x32_10(counter, key, up(out))
    return out


def sample(mean, std, noise, low, high):
    noise = f32(noise)
    B, S, T, A = noise.shape
    out = np.empty_like(noise)
    lib.orc_sample(fp(f32(mean)), fp(f32(std)), fp(noise), fp(f32(low)), fp(f32(high)), B, S, T, A, fp(out))
    return out


def color_noise(noise, beta):
    noise = f32(noise)
    out = np.empty_like(noise)
    lib.orc_color_noise(fp(noise), fp(out), *noise.shape, F(beta))
    return out


def inject_carried(cand, carried, keep):
    cand = f32(cand).copy()
    carried = f32(carried)
    B, S, T, A = cand.shape
    lib.orc_inject_carried(fp(cand), fp(carried), carried.shape[1], keep, B, S, T, A)
    return cand


def mppi_weighted(cand, scores, temperature):
    cand = f32(cand)
    B, S, T, A = cand.shape
    out = np.empty((B, T, A), np.float32)
    lib.orc_mppi_weighted(fp(cand), fp(f32(scores)), B, S, T, A, F(temperature), fp(out))
    return out


def lowest_k(scores, k):
    scores = f32(scores)
    B, S = scores.shape
    out = np.empty((B, k), np.uint32)
    lib.orc_lowest_k(fp(scores), B, S, k, up(out))
    return out


def gather(cand, idx):
    cand = f32(cand)
    idx = np.ascontiguousarray(idx, dtype=np.uint32)
    B, S, T, A = cand.shape
    k = idx.shape[1]
    out = np.empty((B, k, T, A), np.float32)
    lib.orc_gather(fp(cand), up(idx), B, S, k, T, A, fp(out))
    return out


def refit(elites, min_std):
    elites = f32(elites)
    B, k, T, A = elites.shape
    mean = np.empty((B, T, A), np.float32)
    std = np.empty((B, T, A), np.float32)
    lib.orc_refit(fp(elites), B, k, T, A, F(min_std), fp(mean), fp(std))
    return mean, std


def shift(seq):
    seq = f32(seq)
    out = np.empty_like(seq)
    lib.orc_shift(fp(seq), *seq.shape, fp(out))
    return out


def plant_step(domain, state, motors, cmd, dt):
    lib.orc_plant_step(C.byref(_own(Domain, domain)), fp(state), fp(motors), fp(f32(cmd)), F(dt))


def nominal_rollout(initial, actions, motors, dt, substeps, domain, kernel_form=False):
    actions = f32(actions)
    N, T, _ = actions.shape
    out = np.empty((N, T, 18), np.float32)
    fn = lib.orc_nominal_rollout_k4 if kernel_form else lib.orc_nominal_rollout
    fn(fp(f32(initial)), fp(actions), fp(f32(motors)), N, T, F(dt), substeps, C.byref(_own(Domain, domain)), fp(out))
    return out


def tracking_scores(pred, actions, ref_states, ref_actions, cost):
    pred = f32(pred)
    B, S, T, _ = pred.shape
    out = np.empty((B, S), np.float32)
    lib.orc_tracking_scores(fp(pred), fp(f32(actions)), fp(f32(ref_states)), fp(f32(ref_actions)),
                            C.byref(_own(TrackingCost, cost)),
                            B, S, T, fp(out))
    return out


def nominal_scores(initial, motors, ref_states, ref_actions, cost, dt, trim, cand, substeps=10, domain=None,
                   domains=None, with_states=False):
    cand = f32(cand)
    B, S, T, _ = cand.shape
    scores = np.empty((B, S), np.float32)
    states = np.empty((B, S, T, 18), np.float32) if with_states else None
    d = _own(Domain, domain) or Domain.default()
    dd = (Domain * B)(*[_own(Domain, x) for x in domains]) if domains is not None else None
    cost = _own(TrackingCost, cost)
    lib.orc_nominal_scores(fp(f32(initial)), fp(f32(motors)), fp(f32(ref_states)), fp(f32(ref_actions)),
                           C.byref(cost), F(dt), F(trim), substeps, C.byref(d), dd, fp(cand), B, S, T, fp(scores),
                           fp(states))
    return (scores, states) if with_states else scores


class SkyJepaModel:
    """Oracle SkyJEPA model over a weight blob (the layout of include/lewm_b200.h)."""

    def __init__(self, cfg: SkyJepaConfig, weights: np.ndarray, tensor_core_rounding: bool = False):
        """`tensor_core_rounding`: round where the bf16 tensor-core rollout
        rounds (bf16 GRU / first prober-layer weights, combined GRU biases,
        bf16 encoder outputs and GEMM copy of h; f32 state and accumulation)."""
        self.cfg = cfg
        self.weights = f32(weights)
        cfg = _own(SkyJepaConfig, cfg)
        n = lib.orc_skyjepa_weight_count(C.byref(cfg))
        if n != self.weights.size:
            raise ValueError(f"weight blob has {self.weights.size} values, oracle layout needs {n}")
        self.handle = lib.orc_skyjepa_new(C.byref(cfg), fp(self.weights), self.weights.size)
        if tensor_core_rounding:
            lib.orc_skyjepa_set_tensor_core_rounding(self.handle)

    def __del__(self):
        # at interpreter exit the module's `lib` may already be gone
        if getattr(self, "handle", None) and globals().get("lib") is not None:
            lib.orc_skyjepa_free(self.handle)
            self.handle = None

    def tcn_last(self, which: int, x):
        x = f32(x)
        N, time, _ = x.shape
        enc = self.cfg.action_encoder if which else self.cfg.state_encoder
        out = np.empty((N, enc.channels[enc.levels - 1]), np.float32)
        lib.orc_tcn_forward_last(self.handle, which, fp(x), N, time, fp(out))
        return out

    def initial_latent(self, norm_state_hist):
        x = f32(norm_state_hist)
        out = np.empty((x.shape[0], self.cfg.latent_dim), np.float32)
        lib.orc_initial_latent(self.handle, fp(x), x.shape[0], fp(out))
        return out

    def gru_step(self, x, h):
        x, h = f32(x), f32(h)
        out = np.empty_like(h)
        lib.orc_gru_step(self.handle, fp(x), fp(h), h.shape[0], fp(out))
        return out

    def rollout_latents(self, nsh, nah, ncand):
        ncand = f32(ncand)
        B, S, T, _ = ncand.shape
        out = np.empty((B, S, T, self.cfg.latent_dim), np.float32)
        lib.orc_rollout_latents(self.handle, fp(f32(nsh)), fp(f32(nah)), fp(ncand), B, S, T, fp(out))
        return out

    def prober(self, latents):
        lat = f32(latents)
        N = lat.size // self.cfg.latent_dim
        out = np.empty((N, 15), np.float32)
        lib.orc_prober(self.handle, fp(lat), N, fp(out))
        return out

    def scores(self, norm, state_hist, action_hist, ref_states, ref_actions, cost, dt, cand, with_states=False,
               masses=None):
        cand = f32(cand)
        masses = None if masses is None else f32(masses)
        B, S, T, _ = cand.shape
        scores = np.empty((B, S), np.float32)
        states = np.empty((B, S, T, 18), np.float32) if with_states else None
        sm, ss, am, as_ = (f32(v) for v in norm)
        lib.orc_skyjepa_scores(self.handle, fp(sm), fp(ss), fp(am), fp(as_), fp(f32(state_hist)),
                               fp(f32(action_hist)), fp(f32(ref_states)), fp(f32(ref_actions)),
                               C.byref(_own(TrackingCost, cost)), F(dt), fp(cand), B, S, T, fp(masses), fp(scores),
                               fp(states))
        return (scores, states) if with_states else scores

    def score_ctx(self, norm, state_hist, action_hist, ref_states, ref_actions, cost, dt, masses=None):
        cost = _own(TrackingCost, cost)
        keep = [f32(v) for v in norm] + [f32(state_hist), f32(action_hist), f32(ref_states), f32(ref_actions)]
        m = None if masses is None else f32(masses)
        ctx = SkyCtx(self.handle, *(fp(v) for v in keep), cost, dt, fp(m))
        keep.append(m)
        ctx._keep = keep
        return ctx


def integrate(initial, actions, dt, residual, maps, kin, reference_form=False):
    actions = f32(actions)
    N, T, _ = actions.shape
    out = np.empty((N, T, 18), np.float32)
    fn = lib.orc_integrate_reference if reference_form else lib.orc_integrate_k3
    fn(fp(f32(initial)), fp(actions), fp(f32(dt)), fp(f32(residual)), fp(f32(maps)), N, T,
       C.byref(_own(KinematicConfig, kin)), fp(out))
    return out


def so3_exp(w):
    out = np.empty(9, np.float32)
    lib.orc_so3_exp(fp(f32(w)), fp(out))
    return out.reshape(3, 3)


def nominal_ctx(initial, motors, ref_states, ref_actions, cost, dt, trim, substeps=10, domain=None, domains=None):
    keep = [f32(initial), f32(motors), f32(ref_states), f32(ref_actions)]
    dd = (Domain * len(domains))(*[_own(Domain, x) for x in domains]) if domains is not None else None
    ctx = NominalCtx(*(fp(v) for v in keep), _own(TrackingCost, cost), dt, trim, substeps,
                     _own(Domain, domain) or Domain.default(), dd)
    ctx._keep = (keep, dd)
    return ctx


def _plan_common(fn_user, B, S, T, A):
    if isinstance(fn_user, tuple):
        fn, user = fn_user
        return C.cast(fn, VP), C.cast(C.pointer(user), VP), None

    def cb(_user, cand, b, s, t, a, scores):
        c = np.ctypeslib.as_array(cand, shape=(b, s, t, a))
        out = np.ctypeslib.as_array(scores, shape=(b, s))
        out[...] = fn_user(c.copy())
    cfn = SCORE_FN(cb)
    return C.cast(cfn, VP), None, cfn


def mppi_plan(cfg, B, scorer, noise=None, seed=0, offset=0, warm_start=None):
    """scorer: python fn(cand)->scores, or (NOMINAL_FN, NominalCtx) / (SKYJEPA_FN, SkyCtx)."""
    c = _own(_MppiConfig, cfg._c())
    S, T, A = cfg.samples, cfg.horizon, cfg.action_dim
    fnp, user, keep = _plan_common(scorer, B, S, T, A)
    seq = np.empty((B, T, A), np.float32)
    scores = np.empty((B, S), np.float32)
    best = np.empty(B, np.uint32)
    warm = np.empty((B, T, A), np.float32)
    cand = np.empty((B, S, T, A), np.float32)
    lib.orc_mppi_plan(C.byref(c), fp(f32(warm_start)) if warm_start is not None else None, B,
                      fp(f32(noise)) if noise is not None else None, seed, offset, fnp, user, fp(seq), fp(scores),
                      up(best), fp(warm), fp(cand))
    return dict(sequence=seq, scores=scores, best=best, warm=warm, candidates=cand)


def cem_plan(cfg, B, scorer, noise=None, seed=0, offset=0):
    c = _own(_CemConfig, cfg._c())
    S, T, A = cfg.samples, cfg.horizon, cfg.action_dim
    fnp, user, keep = _plan_common(scorer, B, S, T, A)
    seq = np.empty((B, T, A), np.float32)
    scores = np.empty((B, S), np.float32)
    best = np.empty(B, np.uint32)
    cand = np.empty((B, S, T, A), np.float32)
    elites = np.empty((cfg.iterations, B, cfg.elites), np.uint32)
    iter_scores = np.empty((cfg.iterations, B, S), np.float32)
    lib.orc_cem_plan(C.byref(c), B, fp(f32(noise)) if noise is not None else None, seed, offset, fnp, user, fp(seq),
                     fp(scores), up(best), fp(cand), up(elites), fp(iter_scores))
    return dict(sequence=seq, scores=scores, best=best, candidates=cand, elites=elites, iteration_scores=iter_scores)


def icem_plan(cfg, B, scorer, noise=None, seed=0, offset=0, warm_start=None):
    c = _own(_IcemConfig, cfg._c())
    S, T, A = cfg.samples, cfg.horizon, cfg.action_dim
    fnp, user, keep = _plan_common(scorer, B, S, T, A)
    seq = np.empty((B, T, A), np.float32)
    scores = np.empty((B, S), np.float32)
    best = np.empty(B, np.uint32)
    warm = np.empty((B, T, A), np.float32)
    cand = np.empty((B, S, T, A), np.float32)
    elites = np.empty((cfg.iterations, B, cfg.elites), np.uint32)
    iter_scores = np.empty((cfg.iterations, B, S), np.float32)
    lib.orc_icem_plan(C.byref(c), fp(f32(warm_start)) if warm_start is not None else None, B,
                      fp(f32(noise)) if noise is not None else None, seed, offset, fnp, user, fp(seq), fp(scores),
                      up(best), fp(warm), fp(cand), up(elites), fp(iter_scores))
    return dict(sequence=seq, scores=scores, best=best, warm=warm, candidates=cand, elites=elites,
                iteration_scores=iter_scores)


def icem_trace(cfg, B, scorer, noise=None, seed=0, offset=0, warm_start=None):
    c = _own(_IcemConfig, cfg._c())
    S, T, A = cfg.samples, cfg.horizon, cfg.action_dim
    fnp, user, keep = _plan_common(scorer, B, S, T, A)
    seq = np.empty((B, T, A), np.float32)
    scores = np.empty((B, S), np.float32)
    best = np.empty(B, np.uint32)
    warm = np.empty((B, T, A), np.float32)
    trace = np.empty((cfg.iterations, 4, B), np.float32)
    lib.orc_icem_trace(C.byref(c), fp(f32(warm_start)) if warm_start is not None else None, B,
                       fp(f32(noise)) if noise is not None else None, seed, offset, fnp, user, fp(seq), fp(scores),
                       up(best), fp(warm), fp(trace))
    return dict(sequence=seq, scores=scores, best=best, warm=warm, trace=trace)


def reference_state(kind: int, time: float, radius: float, period: float):
    out = np.empty(18, np.float32)
    lib.orc_reference_state(kind, F(time), F(radius), F(period), fp(out))
    return out


def geometric_prior(current, refs, dt, domain=None):
    refs = f32(refs)
    out = np.empty((refs.shape[0], 4), np.float32)
    lib.orc_geometric_prior(fp(f32(current)), fp(refs), refs.shape[0], F(dt), C.byref(_own(Domain, domain) or Domain.default()),
                            fp(out))
    return out


def _media_out(B, oh, ow, history_len, out):
    shape = (B, 3, oh, ow) if history_len == 0 else (B, history_len, 3, oh, ow)
    if out is None:
        return np.zeros(shape, np.float32)
    assert out.shape == shape and out.dtype == np.float32 and out.flags.c_contiguous
    return out


def preprocess_packed(frames, fmt, out_h, out_w, mean=(0, 0, 0), std=(1, 1, 1), history_len=0, slot=0, out=None):
    """frames: u8 [B,H,W,C]; returns f32 [B,3,oh,ow] or [B,history,3,oh,ow]."""
    frames = np.ascontiguousarray(frames, np.uint8)
    B, H, W, _ = frames.shape
    res = _media_out(B, out_h, out_w, history_len, out)
    lib.orc_preprocess_packed(frames.ctypes.data, B, H, W, fmt, out_h, out_w, fp(f32(mean)), fp(f32(std)),
                              history_len, slot, fp(res))
    return res


def preprocess_nv12(y_plane, uv_plane, color_space, out_h, out_w, mean=(0, 0, 0), std=(1, 1, 1), history_len=0,
                    slot=0, out=None):
    """y_plane: u8 [B,H,W]; uv_plane: u8 [B,H/2,W/2,2]."""
    y_plane = np.ascontiguousarray(y_plane, np.uint8)
    uv_plane = np.ascontiguousarray(uv_plane, np.uint8)
    B, H, W = y_plane.shape
    assert uv_plane.shape == (B, H // 2, W // 2, 2)
    res = _media_out(B, out_h, out_w, history_len, out)
    lib.orc_preprocess_nv12(y_plane.ctypes.data, uv_plane.ctypes.data, B, H, W, color_space, out_h, out_w,
                            fp(f32(mean)), fp(f32(std)), history_len, slot, fp(res))
    return res


class LewmCtx(C.Structure):
    _fields_ = [("model", VP), ("emb", FP), ("goal", FP), ("h", U32), ("history", U32)]


LEWM_FN = C.cast(lib.orc_lewm_score_fn, VP)


class LewmModel:
    """orc_lewm: LeWM / WorldModel restated in C (lewm_world.c)."""

    def __init__(self, cfg, weights: np.ndarray):
        self.cfg = cfg
        w = f32(weights)
        self.handle = lib.orc_lewm_new(C.byref(cfg), fp(w), w.size)
        if not self.handle:
            raise ValueError("LeWM weight count mismatch")

    def __del__(self):
        if getattr(self, "handle", None) and globals().get("lib") is not None:
            lib.orc_lewm_free(self.handle)
            self.handle = None

    def action_embed(self, act):
        act = f32(act)
        n = act.size // self.cfg.action_dim
        out = np.empty((n, self.cfg.embed_dim), np.float32)
        lib.orc_lewm_action_embed(self.handle, fp(act), n, fp(out))
        return out

    def predict_last(self, frames, act_emb):
        frames, act_emb = f32(frames), f32(act_emb)
        seqs, t, _ = frames.shape
        out = np.empty((seqs, self.cfg.embed_dim), np.float32)
        lib.orc_lewm_predict_last(self.handle, fp(frames), fp(act_emb), seqs, t, fp(out))
        return out

    def scores(self, emb, goal, cand, history=0, with_last=False):
        emb, goal, cand = f32(emb), f32(goal), f32(cand)
        B, h, _ = emb.shape
        _, S, T, _ = cand.shape
        scores = np.empty((B, S), np.float32)
        last = np.empty((B, S, self.cfg.embed_dim), np.float32) if with_last else None
        lib.orc_lewm_scores(self.handle, fp(emb), h, fp(goal), fp(cand), B, S, T, history or h, fp(scores), fp(last))
        return (scores, last) if with_last else scores

    def encode_vector(self, obs):
        obs = f32(obs)
        out = np.empty((obs.shape[0], self.cfg.embed_dim), np.float32)
        lib.orc_lewm_encode_vector(self.handle, fp(obs), obs.shape[0], fp(out))
        return out

    def encode_pixels(self, pixels):
        pixels = f32(pixels)
        out = np.empty((pixels.shape[0], self.cfg.embed_dim), np.float32)
        lib.orc_lewm_encode_pixels(self.handle, fp(pixels), pixels.shape[0], fp(out))
        return out

    def score_ctx(self, emb, goal, history=0):
        emb, goal = f32(emb), f32(goal)
        ctx = LewmCtx(self.handle, fp(emb), fp(goal), emb.shape[1], history or emb.shape[1])
        ctx._keep = (emb, goal)
        return ctx


# ------------------------------------------------------------ control session

def reference_horizon(kind: int, time: float, dt: float, horizon: int, radius: float, period: float):
    """skyjepa_reference_horizon (src/skyjepa_task.rs:44-55): states at
    time + k dt, k = 1..horizon, in f32."""
    t0, d = np.float32(time), np.float32(dt)
    return np.stack([reference_state(kind, float(t0 + np.float32(k) * d), radius, period)
                     for k in range(1, horizon + 1)])


def shifted_residual(sequence, prior, limit):
    """shifted_residual (src/models/skyjepa/session.rs:534-543)."""
    r = np.clip(f32(sequence) - f32(prior), np.float32(-limit), np.float32(limit)).astype(np.float32)
    out = np.zeros_like(r)
    out[:-1] = r[1:]
    return out


class _SessionPlanner:
    """The session's MppiConfig (SkyJepaControlConfig::mppi_config,
    src/models/skyjepa/control.rs:124-132) as the oracle planner takes it."""

    def __init__(self, cfg, high, hover):
        c = _MppiConfig()
        c.horizon, c.samples, c.iterations, c.action_dim = cfg.horizon, cfg.samples, cfg.iterations, 4
        for i in range(4):
            c.bounds_low[i], c.bounds_high[i] = 0.0, float(high)
            c.noise_std_per_action[i] = cfg.action_noise[i]
            c.deadline_action[i] = float(hover[i])
        c.noise_std = 1.0
        c.has_noise_std_per_action = 1
        c.temperature = cfg.temperature
        c.deadline_ns = -1
        c.has_deadline_action = 1
        c.has_seed, c.seed = 1, cfg.planner_seed
        self.c = c
        self.horizon, self.samples, self.action_dim, self.iterations = cfg.horizon, cfg.samples, 4, cfg.iterations

    def _c(self):
        return self.c


class SkyJepaSession:
    """SkyJepaControllerSession (src/models/skyjepa/session.rs:241-445)
    restated over the oracle's planner, scorers and geometric prior.
    `sky` = (SkyJepaConfig, weights, (state_mean, state_std, action_mean,
    action_std)) for the learned dynamics, None for the nominal physics."""

    def __init__(self, cfg: SessionConfig, initial, sky=None):
        dom = Domain.default()
        cfg = _own(SessionConfig, cfg)
        self.cfg, self.dom = cfg, dom
        self.hover = np.full(4, np.float32(dom.mass) * np.float32(dom.gravity) / np.float32(4.0), np.float32)
        self.high = np.float32(dom.mass) * np.float32(dom.gravity) * np.float32(dom.max_thrust_weight) / np.float32(4.0)
        self.model = None if sky is None else SkyJepaModel(sky[0], sky[1])
        self.norm = None if sky is None else sky[2]
        self.H = sky[0].history_steps if sky is not None else 10
        self.mppi = _SessionPlanner(cfg, self.high, self.hover)
        self.reset_with_action(initial, self.hover)

    def reset_with_action(self, state, action):
        a = f32(action)
        collective = ((a[0] + a[1]) + a[2]) + a[3]
        nominal = ((self.hover[0] + self.hover[1]) + self.hover[2]) + self.hover[3]
        self.trim = collective / nominal * np.float32(self.cfg.trim_multiplier)
        self.motors = (a / self.trim).astype(np.float32)
        self.states = [f32(state).copy() for _ in range(self.H)]
        self.actions = [a.copy() for _ in range(self.H - 1)]
        self.active = self.pending = None
        self.offset = 0  # MppiPlanner::new: a fresh sampler

    def commit_observation(self, state, action):
        self.active, self.pending = self.pending, None
        response = np.float32(1.0) - np.exp(np.float32(-self.cfg.dt) / np.float32(self.dom.motor_time_constant),
                                            dtype=np.float32)
        for i in range(4):
            target = np.clip(np.float32(action[i]) / self.trim, np.float32(0.0), self.high)
            self.motors[i] += (target - self.motors[i]) * response
        self.states = self.states[1:] + [f32(state).copy()]
        self.actions = self.actions[1:] + [f32(action).copy()]

    def plan(self, refs):
        """-> (action sequence [T,4], prior [T,4], best candidate score)."""
        self.pending = None
        refs = f32(refs)
        last = self.states[-1]
        prior = np.clip(geometric_prior(last, refs, self.cfg.dt) * self.trim, 0.0, self.high).astype(np.float32)
        warm = prior + self.active if (self.cfg.warm_start == 1 and self.active is not None) else prior
        warm = np.clip(warm, 0.0, self.high).astype(np.float32)
        if self.model is None:
            c = nominal_ctx(last[None], self.motors[None], refs[None], prior[None], self.cfg.cost, self.cfg.dt,
                            float(self.trim))
            fn = NOMINAL_FN
        else:
            c = self.model.score_ctx(self.norm, np.stack(self.states)[None], np.stack(self.actions)[None],
                                     refs[None], prior[None], self.cfg.cost, self.cfg.dt)
            fn = SKYJEPA_FN
        r = mppi_plan(self.mppi, 1, (fn, c), seed=self.cfg.planner_seed, offset=self.offset, warm_start=warm[None])
        per = self.cfg.samples * self.cfg.horizon * 4
        self.offset += (per + per % 2) * self.cfg.iterations
        if self.cfg.warm_start == 1:
            self.pending = shifted_residual(r["sequence"][0], prior, self.cfg.residual_limit_n)
        return r["sequence"][0], prior, float(r["scores"].min())
