"""Python binding of liblewm_b200.so, the B200 sampling planner.

Mirrors le-wm-nv's planner API (src/planner.rs) and SkyJEPA scorers
(src/models/skyjepa/control.rs) over the C ABI declared in
include/lewm_b200.h: ``MppiPlanner`` / ``CemPlanner`` / ``IcemPlanner`` with
``plan`` and ``plan_device``, warm-start and RNG-offset methods, and the
``NominalScorer``, ``SkyJepaScorer`` and ``CallbackScorer`` candidate scorers.

The shared library is required: importing this module raises ImportError if it
has not been built (``make -C le-wm-nv_b200``).  There is no CPU fallback.
"""
from __future__ import annotations

import atexit
import ctypes as C
import os
import weakref
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblewm_b200.so")
if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: build it with `make -C le-wm-nv_b200`")
lib = C.CDLL(LIB_PATH)

MAX_ACTION_DIM = 16
TCN_MAX_LEVELS = 8
STATUS = {0: "OK", 1: "INVALID_ARGUMENT", 2: "CUDA_ERROR", 3: "DEADLINE", 4: "NCCL_ERROR", 5: "TIMEOUT", 6: "UNSUPPORTED"}

F = C.c_float
U32 = C.c_uint32
U64 = C.c_uint64
I32 = C.c_int32
FP = C.POINTER(C.c_float)
VP = C.c_void_p


class FaultKnobs(C.Structure):
    """lwm_test_faults (include/lewm_b200.h)."""
    _fields_ = [("wait_polls", C.c_uint32), ("tc_skip_h_arrive", C.c_uint32), ("media_skip_row_plus1", C.c_uint32)]


class LwmError(RuntimeError):
    """A failing lwm_* call: .status is the lwm_status name."""

    def __init__(self, status: int, message: str):
        super().__init__(f"{STATUS.get(status, status)}: {message}")
        self.status = STATUS.get(status, str(status))
        self.message = message


# ------------------------------------------------------------------ structs

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
        lib.lwm_domain_default(C.byref(d))
        return d

    @staticmethod
    def sample(seed: int) -> "Domain":
        d = Domain()
        lib.lwm_domain_sample(U64(seed), C.byref(d))
        return d

    def hover_force(self) -> float:
        return float(np.float32(self.mass) * np.float32(self.gravity) / (np.float32(4.0) * np.float32(self.thrust_scale)))


class ImagePreprocess(C.Structure):
    """ImagePreprocess (src/media/mod.rs:168-193)."""
    _fields_ = [("output_height", C.c_uint32), ("output_width", C.c_uint32), ("mean", C.c_float * 3),
                ("std", C.c_float * 3)]

    @classmethod
    def make(cls, output_height: int, output_width: int, mean=(0.0, 0.0, 0.0), std=(1.0, 1.0, 1.0)):
        return cls(output_height, output_width, (C.c_float * 3)(*mean), (C.c_float * 3)(*std))

    @classmethod
    def imagenet_224(cls):
        out = cls()
        lib.lwm_image_preprocess_imagenet_224(C.byref(out))
        return out


class TrackingCost(C.Structure):
    """SkyJepaTrackingCost (src/models/skyjepa/control.rs:19-37)."""
    _fields_ = [("position", F), ("velocity", F), ("attitude", F), ("angular_velocity", F), ("action", F * 4)]

    @staticmethod
    def paper() -> "TrackingCost":
        c = TrackingCost()
        lib.lwm_tracking_cost_paper(C.byref(c))
        return c

    @staticmethod
    def make(position, velocity, attitude, angular_velocity, action) -> "TrackingCost":
        return TrackingCost(position, velocity, attitude, angular_velocity, (F * 4)(*action))


class NominalScorerConfig(C.Structure):
    _fields_ = [("dt", F), ("trim_scale", F), ("substeps", U32), ("cost", TrackingCost), ("domain", Domain)]


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
        lib.lwm_skyjepa_config_paper(C.byref(c))
        return c

    @staticmethod
    def wide() -> "SkyJepaConfig":
        c = SkyJepaConfig()
        lib.lwm_skyjepa_config_wide(C.byref(c))
        return c

    def weight_count(self) -> int:
        return int(lib.lwm_skyjepa_weight_count(C.byref(self)))

    def random_weights(self, seed: int) -> np.ndarray:
        n = self.weight_count()
        if n == 0:
            raise LwmError(1, "invalid SkyJEPA configuration")
        out = np.empty(n, dtype=np.float32)
        _check(lib.lwm_skyjepa_random_weights(C.byref(self), U64(seed), _fp(out), C.c_size_t(n)))
        return out

    def tensors(self) -> List["TensorInfo"]:
        """The weight blob's tensors in order, with their VarBuilder names."""
        n = int(lib.lwm_skyjepa_tensor_info(C.byref(self), 0, None))
        out = []
        for i in range(n):
            t = _TensorInfo()
            lib.lwm_skyjepa_tensor_info(C.byref(self), i, C.byref(t))
            out.append(t.info())
        return out

    def weights_from_safetensors(self, latent_path: str, prober_path: str) -> np.ndarray:
        """The latent model and the prober from their safetensors files
        (SkyJepaSession::open, src/models/skyjepa/session.rs:183-199)."""
        n = self.weight_count()
        out = np.empty(n, dtype=np.float32)
        _check(lib.lwm_skyjepa_weights_from_safetensors(C.byref(self), os.fsencode(latent_path),
                                                        os.fsencode(prober_path), _fp(out), C.c_size_t(n)))
        return out


class LewmConfig(C.Structure):
    """LeWmConfig / WorldModelConfig (src/models/lewm/config.rs, src/models/world_model/config.rs)."""
    _fields_ = [(n, U32) for n in ("embed_dim", "action_dim", "smoothed_dim", "action_mlp_scale", "history_size",
                                   "num_frames", "pred_hidden_dim", "depth", "heads", "dim_head", "mlp_dim",
                                   "pred_proj_hidden")] + \
               [("pred_proj_norm", I32), ("encoder", I32), ("obs_dim", U32), ("obs_hidden_dim", U32),
                ("obs_depth", U32), ("obs_norm", I32), ("image_size", U32), ("patch_size", U32),
                ("vit_hidden", U32), ("vit_layers", U32), ("vit_heads", U32), ("vit_mlp", U32), ("vit_eps", F),
                ("channels", U32), ("qkv_bias", I32), ("projector_hidden", U32), ("projector_norm", I32)]

    @staticmethod
    def vector() -> "LewmConfig":
        c = LewmConfig()
        lib.lwm_lewm_config_vector(C.byref(c))
        return c

    @staticmethod
    def image() -> "LewmConfig":
        c = LewmConfig()
        lib.lwm_lewm_config_image(C.byref(c))
        return c

    def weight_count(self) -> int:
        return int(lib.lwm_lewm_weight_count(C.byref(self)))

    def random_weights(self, seed: int) -> np.ndarray:
        n = self.weight_count()
        if n == 0:
            raise LwmError(1, "invalid LeWM configuration")
        out = np.empty(n, dtype=np.float32)
        _check(lib.lwm_lewm_random_weights(C.byref(self), U64(seed), _fp(out), C.c_size_t(n)))
        return out

    def tensors(self, names: str = "world_model") -> List["TensorInfo"]:
        """The weight blob's tensors in order, named as a LeWm ("lewm") or
        WorldModel ("world_model") checkpoint names them."""
        k = LEWM_NAMES[names]
        n = int(lib.lwm_lewm_tensor_info(C.byref(self), k, 0, None))
        out = []
        for i in range(n):
            t = _TensorInfo()
            lib.lwm_lewm_tensor_info(C.byref(self), k, i, C.byref(t))
            out.append(t.info())
        return out

    def weights_from_safetensors(self, path: str, names: str = "world_model") -> np.ndarray:
        n = self.weight_count()
        out = np.empty(n, dtype=np.float32)
        _check(lib.lwm_lewm_weights_from_safetensors(C.byref(self), LEWM_NAMES[names], os.fsencode(path), _fp(out),
                                                     C.c_size_t(n)))
        return out


LEWM_NAMES = {"lewm": 0, "world_model": 1}
PRECISIONS = {"f32": 0, "bf16": 1, "f32-cuda-core": 2}


@dataclass(frozen=True)
class TensorInfo:
    name: str
    shape: Tuple[int, ...]
    offset: int
    numel: int
    file: int


class _TensorInfo(C.Structure):
    _fields_ = [("name", C.c_char * 160), ("rank", U32), ("shape", U32 * 4), ("offset", C.c_size_t),
                ("numel", C.c_size_t), ("file", I32)]

    def info(self) -> TensorInfo:
        return TensorInfo(self.name.decode(), tuple(int(self.shape[i]) for i in range(self.rank)), int(self.offset),
                          int(self.numel), int(self.file))


NORM_KINDS = {"batch": 0, "layer": 1, "none": 2}


class _PlanResult(C.Structure):
    # the output pointers as plain addresses (filled by _addr, the cheap path)
    _fields_ = [("first_action", VP), ("sequence", VP), ("scores", VP), ("scores_capacity", C.c_size_t),
                ("best_indices", VP), ("batch", U32), ("scores_cols", U32),
                ("iterations_completed", U32), ("elapsed_ns", U64), ("deadline_reached", I32),
                ("deadline_outcome", I32)]


class _PlanDeviceResult(C.Structure):
    _fields_ = [("first_action", VP), ("sequence", VP), ("scores", VP), ("best_indices", VP), ("batch", U32),
                ("scores_cols", U32), ("iterations_completed", U32), ("elapsed_ns", U64),
                ("deadline_reached", I32), ("deadline_outcome", I32)]


class FleetStep(C.Structure):
    """lwm_fleet_step: one control step of a fleet on the device (all pointers device addresses)."""
    _fields_ = [("batch", U32), ("horizon", U32), ("history", U32), ("time", F), ("dt", F), ("reference_kind", I32),
                ("radius", F), ("period", F), ("prior_domain", Domain), ("trim", VP), ("state", VP),
                ("last_action", VP), ("last_action_stride", U32), ("state_history", VP), ("action_history", VP),
                ("reference_states", VP), ("reference_actions", VP)]


SCORE_FN = C.CFUNCTYPE(C.c_int, VP, VP, U32, U32, U32, U32, VP, VP)
EXCHANGE_FN = C.CFUNCTYPE(C.c_int, VP, VP, C.c_size_t, VP, VP)

# ------------------------------------------------------------- signatures

def _sig(name, restype, *argtypes):
    fn = getattr(lib, name)
    fn.restype = restype
    fn.argtypes = list(argtypes)
    return fn


_sig("lwm_last_error", C.c_char_p)
_sig("lwm_version", C.c_char_p)
_sig("lwm_abi_version", C.c_int)
_sig("lwm_ctx_create", C.c_int, C.c_int, C.POINTER(VP))
_sig("lwm_ctx_destroy", C.c_int, VP)
_sig("lwm_ctx_stream", C.c_int, VP, C.POINTER(VP))
_sig("lwm_ctx_synchronize", C.c_int, VP)
_sig("lwm_ctx_launch_count", C.c_int, VP, C.POINTER(U64))
_sig("lwm_ctx_set_kernel_timing", C.c_int, VP, C.c_int)
_sig("lwm_ctx_kernel_time_ms", C.c_int, VP, C.POINTER(C.c_float))
_sig("lwm_mppi_config_default", None, U32, U32, U32, C.POINTER(_MppiConfig))
_sig("lwm_cem_config_default", None, U32, U32, U32, U32, C.POINTER(_CemConfig))
_sig("lwm_icem_config_default", None, U32, U32, U32, U32, C.POINTER(_IcemConfig))
_sig("lwm_mppi_create", C.c_int, VP, C.POINTER(_MppiConfig), C.POINTER(VP))
_sig("lwm_cem_create", C.c_int, VP, C.POINTER(_CemConfig), C.POINTER(VP))
_sig("lwm_icem_create", C.c_int, VP, C.POINTER(_IcemConfig), C.POINTER(VP))
_sig("lwm_planner_destroy", C.c_int, VP)
_sig("lwm_planner_set_warm_start", C.c_int, VP, FP, U32, U32, U32)
_sig("lwm_planner_clear_warm_start", C.c_int, VP)
_sig("lwm_planner_warm_start", C.c_int, VP, FP, C.c_size_t, C.POINTER(U32))
_sig("lwm_planner_reset_rng", C.c_int, VP)
_sig("lwm_planner_rng_offset", C.c_int, VP, C.POINTER(U64))
_sig("lwm_ctx_set_test_faults", C.c_int, VP, C.POINTER(FaultKnobs))
_sig("lwm_planner_elite_indices", C.c_int, VP, C.POINTER(U32), C.c_size_t, C.POINTER(U32), C.POINTER(U32),
     C.POINTER(U32))
_sig("lwm_planner_last_candidates", C.c_int, VP, C.POINTER(VP), C.POINTER(U32))
_sig("lwm_domain_default", None, C.POINTER(Domain))
_sig("lwm_domain_sample", None, U64, C.POINTER(Domain))
_sig("lwm_tracking_cost_paper", None, C.POINTER(TrackingCost))
_sig("lwm_scorer_nominal_create", C.c_int, VP, C.POINTER(NominalScorerConfig), C.POINTER(VP))
_sig("lwm_scorer_nominal_set_context", C.c_int, VP, U32, U32, FP, FP, FP, FP, C.POINTER(Domain))
_sig("lwm_skyjepa_config_paper", None, C.POINTER(SkyJepaConfig))
_sig("lwm_skyjepa_config_wide", None, C.POINTER(SkyJepaConfig))
_sig("lwm_skyjepa_weight_count", C.c_size_t, C.POINTER(SkyJepaConfig))
_sig("lwm_skyjepa_random_weights", C.c_int, C.POINTER(SkyJepaConfig), U64, FP, C.c_size_t)
_sig("lwm_scorer_skyjepa_create", C.c_int, VP, C.POINTER(SkyJepaConfig), FP, C.c_size_t, FP, FP, FP, FP,
     C.POINTER(TrackingCost), F, C.POINTER(VP))
_sig("lwm_scorer_skyjepa_set_context", C.c_int, VP, U32, U32, FP, FP, FP, FP)
_sig("lwm_scorer_skyjepa_set_context_ex", C.c_int, VP, U32, U32, VP, VP, VP, VP, VP)
_sig("lwm_scorer_skyjepa_set_precision", C.c_int, VP, I32)
_sig("lwm_scorer_lewm_set_precision", C.c_int, VP, I32)
_sig("lwm_scorer_callback_create", C.c_int, VP, U32, SCORE_FN, VP, C.POINTER(VP))
_sig("lwm_scorer_score_device", C.c_int, VP, VP, U32, U32, U32, U32, VP)
_sig("lwm_scorer_predict_device", C.c_int, VP, VP, U32, U32, U32, VP)
_sig("lwm_scorer_destroy", C.c_int, VP)
_sig("lwm_plan", C.c_int, VP, VP, VP, C.POINTER(_PlanResult))
_sig("lwm_plan_device", C.c_int, VP, VP, VP, C.POINTER(_PlanDeviceResult))
_sig("lwm_lowest_k_device", C.c_int, VP, VP, U32, U32, U32, VP)
_sig("lwm_color_noise_device", C.c_int, VP, VP, VP, U32, U32, U32, U32, F)
_sig("lwm_normal_device", C.c_int, VP, U64, U64, C.c_size_t, VP)
_sig("lwm_skyjepa_reference_horizon", C.c_int, I32, F, F, U32, F, F, FP)
_sig("lwm_skyjepa_geometric_prior", C.c_int, FP, FP, U32, F, C.POINTER(Domain), FP)
_sig("lwm_rotor_plant_step", C.c_int, C.POINTER(Domain), FP, FP, FP, F)
_sig("lwm_lewm_config_vector", None, C.POINTER(LewmConfig))
_sig("lwm_lewm_config_image", None, C.POINTER(LewmConfig))
_sig("lwm_lewm_weight_count", C.c_size_t, C.POINTER(LewmConfig))
_sig("lwm_lewm_random_weights", C.c_int, C.POINTER(LewmConfig), U64, FP, C.c_size_t)
_sig("lwm_scorer_lewm_create", C.c_int, VP, C.POINTER(LewmConfig), FP, C.c_size_t, C.POINTER(VP))
_sig("lwm_scorer_lewm_set_context", C.c_int, VP, U32, U32, U32, FP, FP)
_sig("lwm_scorer_lewm_set_context_device", C.c_int, VP, U32, U32, U32, VP, VP)
_sig("lwm_lewm_encode_vector_device", C.c_int, VP, VP, U32, VP)
_sig("lwm_lewm_encode_pixels_device", C.c_int, VP, VP, U32, VP)
_sig("lwm_icem_trace_device", C.c_int, VP, VP, VP, C.POINTER(_PlanDeviceResult), C.POINTER(VP))
_sig("lwm_planner_set_shard", C.c_int, VP, U32, U32)
_sig("lwm_plan_device_shard", C.c_int, VP, VP, VP, C.POINTER(VP), C.POINTER(U32))
_sig("lwm_mppi_combine_device", C.c_int, VP, VP, U32, C.POINTER(_PlanDeviceResult))
_sig("lwm_planner_set_shard_exchange", C.c_int, VP, U32, EXCHANGE_FN, VP)
_sig("lwm_fleet_control_step_device", C.c_int, VP, C.POINTER(FleetStep))
_sig("lwm_rotor_plant_step_device", C.c_int, VP, VP, VP, VP, VP, U32, U32, F, U32)
_sig("lwm_scorer_skyjepa_context_device", C.c_int, VP, C.POINTER(VP), C.POINTER(VP), C.POINTER(VP), C.POINTER(VP))
_sig("lwm_planner_set_warm_start_device", C.c_int, VP, VP, U32, U32, U32)
_sig("lwm_skyjepa_tensor_info", C.c_size_t, C.POINTER(SkyJepaConfig), C.c_size_t, C.POINTER(_TensorInfo))
_sig("lwm_lewm_tensor_info", C.c_size_t, C.POINTER(LewmConfig), I32, C.c_size_t, C.POINTER(_TensorInfo))
_sig("lwm_skyjepa_weights_from_safetensors", C.c_int, C.POINTER(SkyJepaConfig), C.c_char_p, C.c_char_p, FP,
     C.c_size_t)
_sig("lwm_lewm_weights_from_safetensors", C.c_int, C.POINTER(LewmConfig), I32, C.c_char_p, FP, C.c_size_t)
_sig("lwm_skyjepa_session_config_paper", None, VP)
_sig("lwm_skyjepa_session_create", C.c_int, VP, VP, VP, FP, C.c_size_t, FP, FP, FP, FP, FP, C.POINTER(VP))
_sig("lwm_skyjepa_session_destroy", None, VP)
_sig("lwm_skyjepa_session_reset", C.c_int, VP, FP)
_sig("lwm_skyjepa_session_reset_with_action", C.c_int, VP, FP, FP)
_sig("lwm_skyjepa_session_commit_observation", C.c_int, VP, FP, FP)
_sig("lwm_skyjepa_session_plan", C.c_int, VP, FP, I32, VP)
_sig("lwm_skyjepa_session_scorer", VP, VP)
_sig("lwm_skyjepa_session_trim_scale", F, VP)
_sig("lwm_skyjepa_shifted_residual", C.c_int, FP, FP, U32, U32, F, FP)
_sig("lwm_image_preprocess_imagenet_224", None, C.POINTER(ImagePreprocess))
_sig("lwm_preprocess_packed_device", C.c_int, VP, VP, U32, U32, U32, I32, C.POINTER(ImagePreprocess), U32, U32, I32,
     VP)
_sig("lwm_preprocess_nv12_device", C.c_int, VP, VP, VP, U32, U32, U32, I32, C.POINTER(ImagePreprocess), U32, U32,
     I32, VP)
_sig("lwm_preprocess_packed_patches_device", C.c_int, VP, VP, U32, U32, U32, I32, C.POINTER(ImagePreprocess), U32,
     I32, VP)
_sig("lwm_preprocess_nv12_patches_device", C.c_int, VP, VP, VP, U32, U32, U32, I32, C.POINTER(ImagePreprocess), U32,
     I32, VP)
_sig("lwm_lewm_encode_nv12_device", C.c_int, VP, VP, VP, U32, U32, U32, I32, C.POINTER(ImagePreprocess), VP)
_sig("lwm_lewm_plan_nv12_device", C.c_int, VP, VP, VP, VP, U32, U32, U32, U32, I32, C.POINTER(ImagePreprocess), VP,
     C.POINTER(_PlanDeviceResult))
_sig("lwm_lewm_encode_packed_device", C.c_int, VP, VP, U32, U32, U32, I32, C.POINTER(ImagePreprocess), VP)


def _check(status: int) -> None:
    if status != 0:
        raise LwmError(status, lib.lwm_last_error().decode())


def _fp(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(FP)


def _addr(a: Optional[np.ndarray]) -> Optional[int]:
    """The address of a C-contiguous array's data for c_void_p arguments: a
    view of its buffer for writable arrays (about a fifth of the cost of
    ndarray.ctypes), ndarray.ctypes.data otherwise."""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    if a.flags["WRITEABLE"] and a.nbytes:
        return C.addressof(C.c_char.from_buffer(a))
    return a.ctypes.data


def _f32(x, shape=None) -> np.ndarray:
    a = np.ascontiguousarray(np.asarray(x, dtype=np.float32))
    if shape is not None:
        a = a.reshape(shape)
    return a


def version() -> str:
    return lib.lwm_version().decode()


# Handles still alive at interpreter exit are released in dependency order
# (planners and scorers before the contexts they use), before the CUDA
# runtime is torn down.
_LIVE = {"planner": weakref.WeakSet(), "scorer": weakref.WeakSet(), "ctx": weakref.WeakSet()}


@atexit.register
def _close_all() -> None:
    for kind in ("planner", "scorer", "ctx"):
        for obj in list(_LIVE[kind]):
            try:
                obj.close()
            except Exception:
                pass


# ------------------------------------------------------------------- context

class Context:
    """A CUDA device and stream (Device::new_cuda, src/runtime.rs:7-18)."""

    def __init__(self, device: int = 0):
        h = VP()
        _check(lib.lwm_ctx_create(device, C.byref(h)))
        self.handle = h
        self.device = device
        _LIVE["ctx"].add(self)

    @property
    def stream(self) -> int:
        s = VP()
        _check(lib.lwm_ctx_stream(self.handle, C.byref(s)))
        return int(s.value or 0)

    def synchronize(self) -> None:
        _check(lib.lwm_ctx_synchronize(self.handle))

    def set_test_faults(self, wait_polls: int = 0, tc_skip_h_arrive: bool = False,
                        media_skip_row: Optional[int] = None) -> None:
        """Fault injection for failure-path tests (lwm_ctx_set_test_faults);
        no arguments clears every knob."""
        f = FaultKnobs(wait_polls, int(tc_skip_h_arrive), 0 if media_skip_row is None else media_skip_row + 1)
        _check(lib.lwm_ctx_set_test_faults(self.handle, C.byref(f)))

    def launch_count(self) -> int:
        n = U64()
        _check(lib.lwm_ctx_launch_count(self.handle, C.byref(n)))
        return int(n.value)

    def set_kernel_timing(self, on: bool = True) -> None:
        """Records CUDA events around every SkyJEPA rollout launch
        (lwm_ctx_set_kernel_timing)."""
        _check(lib.lwm_ctx_set_kernel_timing(self.handle, int(on)))

    def kernel_time_ms(self) -> float:
        """Device time of the last timed rollout launch (lwm_ctx_kernel_time_ms)."""
        ms = C.c_float()
        _check(lib.lwm_ctx_kernel_time_ms(self.handle, C.byref(ms)))
        return float(ms.value)

    def torch_stream(self):
        import torch
        return torch.cuda.ExternalStream(self.stream, device=torch.device("cuda", self.device))

    def close(self) -> None:
        if getattr(self, "handle", None):
            for kind in ("planner", "scorer"):
                for obj in list(_LIVE[kind]):
                    if getattr(obj, "ctx", None) is self:
                        obj.close()
            lib.lwm_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------------- configs

def _bounds(arr, action_dim, default):
    out = (F * MAX_ACTION_DIM)()
    vals = list(arr) if arr is not None else [default] * action_dim
    for i, v in enumerate(vals[:MAX_ACTION_DIM]):
        out[i] = v
    return out


@dataclass
class ActionBounds:
    """ActionBounds (src/planner.rs:67-83)."""
    low: List[float]
    high: List[float]

    @staticmethod
    def symmetric(action_dim: int, limit: float) -> "ActionBounds":
        return ActionBounds([-limit] * action_dim, [limit] * action_dim)

    @staticmethod
    def scalar(action_dim: int, low: float, high: float) -> "ActionBounds":
        return ActionBounds([low] * action_dim, [high] * action_dim)


@dataclass
class MppiConfig:
    """MppiConfig (src/planner.rs:178-208); deadline in seconds."""
    horizon: int
    samples: int
    action_dim: int
    iterations: int = 1
    action_bounds: Optional[ActionBounds] = None
    noise_std: float = 1.0
    noise_std_per_action: Optional[Sequence[float]] = None
    temperature: float = 1.0
    deadline: Optional[float] = None
    deadline_action: Optional[Sequence[float]] = None
    seed: Optional[int] = None

    def _c(self) -> _MppiConfig:
        c = _MppiConfig()
        lib.lwm_mppi_config_default(self.horizon, self.samples, self.action_dim, C.byref(c))
        c.iterations = self.iterations
        b = self.action_bounds or ActionBounds.symmetric(self.action_dim, 1.0)
        c.bounds_low = _bounds(b.low, self.action_dim, -1.0)
        c.bounds_high = _bounds(b.high, self.action_dim, 1.0)
        c.noise_std = self.noise_std
        if self.noise_std_per_action is not None:
            if len(self.noise_std_per_action) != self.action_dim:
                raise LwmError(1, f"MPPI per-action noise length {len(self.noise_std_per_action)} must match "
                                  f"action_dim {self.action_dim}")
            c.has_noise_std_per_action = 1
            c.noise_std_per_action = _bounds(self.noise_std_per_action, self.action_dim, 1.0)
        c.temperature = self.temperature
        c.deadline_ns = -1 if self.deadline is None else int(self.deadline * 1e9)
        if self.deadline_action is not None:
            if len(self.deadline_action) != self.action_dim:
                raise LwmError(1, f"MPPI deadline_action length {len(self.deadline_action)} must match "
                                  f"action_dim {self.action_dim}")
            c.has_deadline_action = 1
            c.deadline_action = _bounds(self.deadline_action, self.action_dim, 0.0)
        if self.seed is not None:
            c.has_seed = 1
            c.seed = self.seed
        return c


@dataclass
class CemConfig:
    """CemConfig (src/planner.rs:107-137)."""
    horizon: int
    samples: int
    elites: int
    action_dim: int
    iterations: int = 4
    action_bounds: Optional[ActionBounds] = None
    init_std: float = 1.0
    min_std: float = 1e-3
    deadline: Optional[float] = None
    deadline_action: Optional[Sequence[float]] = None
    seed: Optional[int] = None

    def _c(self) -> _CemConfig:
        c = _CemConfig()
        lib.lwm_cem_config_default(self.horizon, self.samples, self.elites, self.action_dim, C.byref(c))
        c.iterations = self.iterations
        b = self.action_bounds or ActionBounds.symmetric(self.action_dim, 1.0)
        c.bounds_low = _bounds(b.low, self.action_dim, -1.0)
        c.bounds_high = _bounds(b.high, self.action_dim, 1.0)
        c.init_std = self.init_std
        c.min_std = self.min_std
        c.deadline_ns = -1 if self.deadline is None else int(self.deadline * 1e9)
        if self.deadline_action is not None:
            c.has_deadline_action = 1
            c.deadline_action = _bounds(self.deadline_action, self.action_dim, 0.0)
        if self.seed is not None:
            c.has_seed = 1
            c.seed = self.seed
        return c


@dataclass
class IcemConfig:
    """IcemConfig (src/planner.rs:256-295)."""
    horizon: int
    samples: int
    elites: int
    action_dim: int
    keep_elites: Optional[int] = None
    iterations: int = 4
    noise_beta: float = 2.0
    alpha: float = 0.1
    action_bounds: Optional[ActionBounds] = None
    init_std: float = 1.0
    min_std: float = 1e-3
    return_mean: bool = True
    deadline: Optional[float] = None
    deadline_action: Optional[Sequence[float]] = None
    seed: Optional[int] = None

    def _c(self) -> _IcemConfig:
        c = _IcemConfig()
        lib.lwm_icem_config_default(self.horizon, self.samples, self.elites, self.action_dim, C.byref(c))
        c.keep_elites = self.elites if self.keep_elites is None else self.keep_elites
        c.iterations = self.iterations
        c.noise_beta = self.noise_beta
        c.alpha = self.alpha
        b = self.action_bounds or ActionBounds.symmetric(self.action_dim, 1.0)
        c.bounds_low = _bounds(b.low, self.action_dim, -1.0)
        c.bounds_high = _bounds(b.high, self.action_dim, 1.0)
        c.init_std = self.init_std
        c.min_std = self.min_std
        c.return_mean = 1 if self.return_mean else 0
        c.deadline_ns = -1 if self.deadline is None else int(self.deadline * 1e9)
        if self.deadline_action is not None:
            c.has_deadline_action = 1
            c.deadline_action = _bounds(self.deadline_action, self.action_dim, 0.0)
        if self.seed is not None:
            c.has_seed = 1
            c.seed = self.seed
        return c


# ------------------------------------------------------------------- results

@dataclass
class PlanResult:
    """PlanResult (src/planner.rs:355-366) as numpy arrays."""
    first_action: np.ndarray
    sequence: np.ndarray
    scores: np.ndarray
    best_indices: List[int]
    iterations_completed: int
    elapsed: float
    deadline_reached: bool
    deadline_outcome: str


@dataclass
class PlanDeviceResult:
    """PlanDeviceResult (src/planner.rs:368-379): device addresses owned by the
    planner, valid until its next plan call."""
    first_action: int
    sequence: int
    scores: int
    best_indices: int
    batch: int
    scores_cols: int
    iterations_completed: int
    elapsed: float
    deadline_reached: bool
    deadline_outcome: str


_OUTCOME = {0: "None", 1: "WarmStart", 2: "ConfiguredAction"}


# ------------------------------------------------------------------- scorers

class Scorer:
    handle = None
    batch = 0
    ctx: Context

    def score_device(self, candidates_ptr: int, batch: int, samples: int, horizon: int, action_dim: int,
                     scores_ptr: int) -> None:
        _check(lib.lwm_scorer_score_device(self.handle, VP(candidates_ptr), batch, samples, horizon, action_dim,
                                           VP(scores_ptr)))

    def predict_device(self, candidates_ptr: int, batch: int, samples: int, horizon: int, states_ptr: int) -> None:
        _check(lib.lwm_scorer_predict_device(self.handle, VP(candidates_ptr), batch, samples, horizon,
                                             VP(states_ptr)))

    def close(self) -> None:
        if getattr(self, "handle", None):
            if getattr(self.ctx, "handle", None):
                lib.lwm_scorer_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class NominalScorer(Scorer):
    """SkyJepaNominalScorer (src/models/skyjepa/control.rs:332-428)."""

    def __init__(self, ctx: Context, dt: float, trim_scale: float, cost: TrackingCost, substeps: int = 10,
                 domain: Optional[Domain] = None):
        self.ctx = ctx
        cfg = NominalScorerConfig(dt, trim_scale, substeps, cost, domain or Domain.default())
        h = VP()
        _check(lib.lwm_scorer_nominal_create(ctx.handle, C.byref(cfg), C.byref(h)))
        self.handle = h
        _LIVE["scorer"].add(self)

    def set_context(self, initial, motors, reference_states, reference_actions, domains=None) -> None:
        initial = _f32(initial)
        B = initial.shape[0]
        ref = _f32(reference_states)
        T = ref.shape[1]
        dom = None
        if domains is not None:
            dom = (Domain * B)(*domains)
        _check(lib.lwm_scorer_nominal_set_context(self.handle, B, T, _fp(initial), _fp(_f32(motors)), _fp(ref),
                                                  _fp(_f32(reference_actions)), dom))
        self.batch = B


class SkyJepaScorer(Scorer):
    """SkyJepaMppiScorer (src/models/skyjepa/control.rs:146-317)."""

    def __init__(self, ctx: Context, config: SkyJepaConfig, weights: np.ndarray, state_mean, state_std,
                 action_mean, action_std, cost: TrackingCost, dt: float):
        self.ctx = ctx
        self.config = config
        w = _f32(weights)
        h = VP()
        _check(lib.lwm_scorer_skyjepa_create(ctx.handle, C.byref(config), _fp(w), C.c_size_t(w.size),
                                             _fp(_f32(state_mean)), _fp(_f32(state_std)), _fp(_f32(action_mean)),
                                             _fp(_f32(action_std)), C.byref(cost), F(dt), C.byref(h)))
        self.handle = h
        _LIVE["scorer"].add(self)

    def set_precision(self, precision: str) -> None:
        """"f32" (split-fp16 tensor cores where the shape allows, else CUDA cores; f32-class results),
        "bf16" (bf16 tensor cores where the shape allows) or "f32-cuda-core"."""
        _check(lib.lwm_scorer_skyjepa_set_precision(self.handle, PRECISIONS[precision]))

    def context_device(self):
        """Device addresses (state_history, action_history, reference_states, reference_actions) of the context."""
        ptrs = [VP() for _ in range(4)]
        _check(lib.lwm_scorer_skyjepa_context_device(self.handle, *(C.byref(p) for p in ptrs)))
        return tuple(int(p.value) for p in ptrs)

    def set_context(self, state_history, action_history, reference_states, reference_actions,
                    vehicle_mass=None) -> None:
        """Per-plan context; `vehicle_mass` [B] overrides kinematics.mass per vehicle."""
        sh = _f32(state_history)
        ref = _f32(reference_states)
        m = None if vehicle_mass is None else _f32(vehicle_mass)
        _check(lib.lwm_scorer_skyjepa_set_context_ex(self.handle, sh.shape[0], ref.shape[1], _addr(sh),
                                                     _addr(_f32(action_history)), _addr(ref),
                                                     _addr(_f32(reference_actions)), _addr(m)))
        self.batch = sh.shape[0]


class LewmScorer(Scorer):
    """LeWmSession::score_candidates (src/session.rs:46-66) over a LeWM /
    WorldModel: goal-embedding L2 cost of the rolled-out embeddings."""

    def __init__(self, ctx: Context, config: LewmConfig, weights: np.ndarray):
        self.ctx = ctx
        self.config = config
        w = _f32(weights)
        h = VP()
        _check(lib.lwm_scorer_lewm_create(ctx.handle, C.byref(config), _fp(w), C.c_size_t(w.size), C.byref(h)))
        self.handle = h
        _LIVE["scorer"].add(self)

    def set_precision(self, precision: str) -> None:
        """"f32" (default) or "bf16": the GEMMs on the tcgen05 tensor cores
        with bf16 weights and inputs, f32 accumulation and activations."""
        _check(lib.lwm_scorer_lewm_set_precision(self.handle, PRECISIONS[precision]))

    def set_context(self, emb_history, goal, history: int = 0) -> None:
        """emb_history [B, h, D] and goal [B, D] host arrays; history 0 = h (the session's window)."""
        e = _f32(emb_history)
        _check(lib.lwm_scorer_lewm_set_context(self.handle, e.shape[0], e.shape[1], history, _fp(e),
                                               _fp(_f32(goal))))
        self.batch = e.shape[0]

    def set_context_device(self, emb_history, goal, history: int = 0) -> None:
        """torch CUDA tensors emb_history [B, h, D], goal [B, D] (copied on the context stream)."""
        _check(lib.lwm_scorer_lewm_set_context_device(self.handle, emb_history.shape[0], emb_history.shape[1],
                                                      history, VP(emb_history.data_ptr()), VP(goal.data_ptr())))
        self.batch = emb_history.shape[0]

    def encode_vector(self, obs):
        """WorldModel::encode_vector: torch CUDA [n, obs_dim] -> [n, D] (on the context stream)."""
        import torch
        out = torch.empty((obs.shape[0], self.config.embed_dim), device=obs.device, dtype=torch.float32)
        _check(lib.lwm_lewm_encode_vector_device(self.handle, VP(obs.data_ptr()), obs.shape[0],
                                                 VP(out.data_ptr())))
        return out

    def encode_pixels(self, pixels):
        """LeWm::encode_pixels: torch CUDA [n, C, H, W] normalised -> [n, D] (on the context stream)."""
        import torch
        out = torch.empty((pixels.shape[0], self.config.embed_dim), device=pixels.device, dtype=torch.float32)
        _check(lib.lwm_lewm_encode_pixels_device(self.handle, VP(pixels.data_ptr()), pixels.shape[0],
                                                 VP(out.data_ptr())))
        return out

    def encode_nv12(self, y_plane, uv_plane, n: int, height: int, width: int, color_space, cfg: "ImagePreprocess"):
        """NV12 device frames -> [n, D] embeddings, preprocessed straight into the ViT's patch matrix."""
        import torch
        cs = NV12_COLOR_SPACES[color_space] if isinstance(color_space, str) else int(color_space)
        out = torch.empty((n, self.config.embed_dim), device="cuda", dtype=torch.float32)
        _check(lib.lwm_lewm_encode_nv12_device(self.handle, VP(_ptr(y_plane)), VP(_ptr(uv_plane)), n, height, width,
                                               cs, C.byref(cfg), VP(out.data_ptr())))
        return out

    def encode_packed(self, frames, n: int, height: int, width: int, fmt, cfg: "ImagePreprocess"):
        """Packed RGB/BGR(A) device frames -> [n, D] embeddings, preprocessed straight into the patch matrix."""
        import torch
        f = PACKED_FORMATS[fmt] if isinstance(fmt, str) else int(fmt)
        out = torch.empty((n, self.config.embed_dim), device="cuda", dtype=torch.float32)
        _check(lib.lwm_lewm_encode_packed_device(self.handle, VP(_ptr(frames)), n, height, width, f, C.byref(cfg),
                                                 VP(out.data_ptr())))
        return out


class _CudaArray:
    def __init__(self, ptr: int, shape, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def device_tensor(ptr: int, shape, dtype: str = "f4"):
    """A torch view of device memory owned by the library (no copy)."""
    import torch
    return torch.as_tensor(_CudaArray(ptr, shape, "<" + dtype), device="cuda")


class CallbackScorer(Scorer):
    """The CandidateScorer trait (src/planner.rs:25-32) implemented by a
    Python callable ``fn(candidates: torch.Tensor[B,S,T,A]) -> torch.Tensor[B,S]``
    that runs on the context stream."""

    def __init__(self, ctx: Context, batch: int, fn: Callable):
        import torch
        self.ctx = ctx
        self.batch = batch
        self._fn = fn

        def trampoline(user, cand, B, S, T, A, scores, stream):
            try:
                with torch.cuda.stream(torch.cuda.ExternalStream(stream)):
                    cands = device_tensor(cand, (B, S, T, A))
                    out = device_tensor(scores, (B, S))
                    out.copy_(fn(cands).reshape(B, S).to(torch.float32))
                return 0
            except Exception as exc:  # surfaced as LwmError by the caller
                self.error = exc
                return 1

        self._cb = SCORE_FN(trampoline)
        h = VP()
        _check(lib.lwm_scorer_callback_create(ctx.handle, batch, self._cb, None, C.byref(h)))
        self.handle = h
        _LIVE["scorer"].add(self)


# ------------------------------------------------------------------- planners

class _Planner:
    kind = ""

    def __init__(self, ctx: Context, config):
        self.ctx = ctx
        self.config = config
        self._cfg = config._c()
        h = VP()
        _check(self._create(ctx.handle, C.byref(self._cfg), C.byref(h)))
        self.handle = h
        _LIVE["planner"].add(self)

    def plan(self, scorer: Scorer, injected_noise: Optional[np.ndarray] = None, batch: Optional[int] = None) -> PlanResult:
        cfg = self.config
        B = batch or scorer.batch
        T, A, S = cfg.horizon, cfg.action_dim, cfg.samples
        fa = np.empty((B, A), np.float32)
        seq = np.empty((B, T, A), np.float32)
        sc = np.empty((B, S), np.float32)
        best = np.empty((B,), np.uint32)
        r = _PlanResult(_addr(fa), _addr(seq), _addr(sc), sc.size, _addr(best))
        noise = None if injected_noise is None else _f32(injected_noise)
        _check(lib.lwm_plan(self.handle, scorer.handle, _addr(noise), C.byref(r)))
        cols = r.scores_cols
        scores = sc if cols == S else sc.reshape(-1)[: B * cols].reshape(B, cols).copy()
        return PlanResult(fa, seq, scores, best.tolist(), int(r.iterations_completed), r.elapsed_ns * 1e-9,
                          bool(r.deadline_reached), _OUTCOME[r.deadline_outcome])

    def plan_device(self, scorer: Scorer, injected_noise_ptr: Optional[int] = None) -> PlanDeviceResult:
        r = _PlanDeviceResult()
        _check(lib.lwm_plan_device(self.handle, scorer.handle, VP(injected_noise_ptr) if injected_noise_ptr else None,
                                   C.byref(r)))
        return PlanDeviceResult(r.first_action or 0, r.sequence or 0, r.scores or 0, r.best_indices or 0, r.batch,
                                r.scores_cols, r.iterations_completed, r.elapsed_ns * 1e-9, bool(r.deadline_reached),
                                _OUTCOME[r.deadline_outcome])

    def plan_nv12_device(self, scorer: "LewmScorer", y_plane, uv_plane, batch: int, history: int, height: int,
                         width: int, color_space, cfg: "ImagePreprocess",
                         injected_noise_ptr: Optional[int] = None) -> PlanDeviceResult:
        """One LeWmSession control step (src/session.rs:31-65) on device NV12
        frames: frames [0, batch*history) are the observation history,
        [batch*history, batch*(history+1)) the goals.  Equal to encode_nv12 +
        set_context_device + plan_device, with the frames' encoder running
        beside sampling and the candidate-only part of scoring."""
        cs = NV12_COLOR_SPACES[color_space] if isinstance(color_space, str) else int(color_space)
        r = _PlanDeviceResult()
        _check(lib.lwm_lewm_plan_nv12_device(self.handle, scorer.handle, VP(_ptr(y_plane)), VP(_ptr(uv_plane)), batch,
                                             history, height, width, cs, C.byref(cfg),
                                             VP(injected_noise_ptr) if injected_noise_ptr else None, C.byref(r)))
        scorer.batch = batch
        return PlanDeviceResult(r.first_action or 0, r.sequence or 0, r.scores or 0, r.best_indices or 0, r.batch,
                                r.scores_cols, r.iterations_completed, r.elapsed_ns * 1e-9, bool(r.deadline_reached),
                                _OUTCOME[r.deadline_outcome])

    def set_warm_start_device(self, ptr: int, batch: int) -> None:
        """The warm start from device memory [batch, horizon, action_dim] (on the context stream)."""
        _check(lib.lwm_planner_set_warm_start_device(self.handle, VP(ptr), batch, self.config.horizon,
                                                     self.config.action_dim))

    # ------------------------------------------------ candidate-range shards
    def set_shard(self, sample_base: int, sample_total: int) -> None:
        """Own samples [sample_base, sample_base + samples) of sample_total (0: unsharded)."""
        _check(lib.lwm_planner_set_shard(self.handle, sample_base, sample_total))

    def plan_device_shard(self, scorer: Scorer, injected_noise_ptr: Optional[int] = None):
        """Score this shard; returns (device address of the [B, width] tuples, width)."""
        t = VP()
        w = U32()
        _check(lib.lwm_plan_device_shard(self.handle, scorer.handle,
                                         VP(injected_noise_ptr) if injected_noise_ptr else None, C.byref(t),
                                         C.byref(w)))
        return int(t.value), int(w.value)

    def combine_device(self, tuples_ptr: int, shards: int) -> PlanDeviceResult:
        """Finish the plan from the gathered tuples [shards, B, width] of every shard."""
        r = _PlanDeviceResult()
        _check(lib.lwm_mppi_combine_device(self.handle, VP(tuples_ptr), shards, C.byref(r)))
        return PlanDeviceResult(r.first_action or 0, r.sequence or 0, r.scores or 0, r.best_indices or 0, r.batch,
                                r.scores_cols, r.iterations_completed, r.elapsed_ns * 1e-9, bool(r.deadline_reached),
                                _OUTCOME[r.deadline_outcome])

    def set_shard_exchange(self, shards: int, exchange: Optional[Callable[[int, int, int, int], None]]) -> None:
        """CEM / iCEM shards: `exchange(local_ptr, count, gathered_ptr, stream)`
        all-gathers `count` floats of device memory from every shard (in
        sample-range order) into `gathered_ptr`, on `stream`.  None clears it."""
        if exchange is None:
            self._exchange_cb = None
            _check(lib.lwm_planner_set_shard_exchange(self.handle, 0, None, None))
            return

        def call(_user, local, count, gathered, stream):
            try:
                exchange(int(local or 0), int(count), int(gathered or 0), int(stream or 0))
                return 0
            except Exception:  # reported to the planner as a failed exchange
                import traceback
                traceback.print_exc()
                return 1
        self._exchange_cb = EXCHANGE_FN(call)
        _check(lib.lwm_planner_set_shard_exchange(self.handle, shards, self._exchange_cb, None))

    def last_candidates_ptr(self) -> int:
        p = VP()
        s = U32()
        _check(lib.lwm_planner_last_candidates(self.handle, C.byref(p), C.byref(s)))
        return int(p.value)

    def set_warm_start_sequence(self, sequence) -> None:
        seq = _f32(sequence)
        if seq.ndim != 3:
            raise LwmError(1, f"{self.kind} warm-start must be [batch, horizon, action_dim], got {list(seq.shape)}")
        _check(lib.lwm_planner_set_warm_start(self.handle, _fp(seq), seq.shape[0], seq.shape[1], seq.shape[2]))

    def clear_warm_start(self) -> None:
        _check(lib.lwm_planner_clear_warm_start(self.handle))

    def warm_start_sequence(self, max_batch: int = 4096) -> Optional[np.ndarray]:
        cfg = self.config
        buf = np.empty((max_batch, cfg.horizon, cfg.action_dim), np.float32)
        b = U32()
        _check(lib.lwm_planner_warm_start(self.handle, _fp(buf), C.c_size_t(buf.size), C.byref(b)))
        return None if b.value == 0 else buf[: b.value].copy()

    def reset_rng_sequence(self) -> None:
        _check(lib.lwm_planner_reset_rng(self.handle))

    def rng_offset(self) -> int:
        o = U64()
        _check(lib.lwm_planner_rng_offset(self.handle, C.byref(o)))
        return int(o.value)

    def close(self) -> None:
        if getattr(self, "handle", None):
            if getattr(self.ctx, "handle", None):
                lib.lwm_planner_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class MppiPlanner(_Planner):
    """MppiPlanner (src/planner.rs:544-729)."""
    kind = "MPPI"
    _create = staticmethod(lib.lwm_mppi_create)


class _ElitePlanner(_Planner):
    def elite_indices(self) -> np.ndarray:
        """The elite indices every iteration of the last plan selected, in
        selection order (ascending score, ties to the lower index), as
        [iterations, batch, elites] uint32."""
        its, b, k = U32(), U32(), U32()
        cfg = self.config
        cap = cfg.iterations * 4096 * cfg.elites
        buf = np.empty(cap, np.uint32)
        _check(lib.lwm_planner_elite_indices(self.handle, buf.ctypes.data_as(C.POINTER(U32)), C.c_size_t(cap),
                                             C.byref(its), C.byref(b), C.byref(k)))
        n = its.value * b.value * k.value
        return buf[:n].reshape(its.value, b.value, k.value).copy()


class CemPlanner(_ElitePlanner):
    """CemPlanner (src/planner.rs:418-541)."""
    kind = "CEM"
    _create = staticmethod(lib.lwm_cem_create)

    def set_warm_start_sequence(self, sequence) -> None:  # CEM has no warm start in the reference
        raise LwmError(1, "CEM planners have no warm start")


class IcemPlanner(_ElitePlanner):
    """IcemPlanner (src/planner.rs:731-1053)."""
    kind = "iCEM"
    _create = staticmethod(lib.lwm_icem_create)

    def trace_device(self, scorer: Scorer, injected_noise_ptr: Optional[int] = None):
        """IcemPlanner::trace_device (src/planner.rs:900-1010): the plan plus, per
        iteration, [mean_score, best_candidate_score, elite_mean_score,
        updated_mean_score] per vehicle, as a host array [iterations, 4, B]."""
        r = _PlanDeviceResult()
        t = VP()
        _check(lib.lwm_icem_trace_device(self.handle, scorer.handle,
                                         VP(injected_noise_ptr) if injected_noise_ptr else None, C.byref(r),
                                         C.byref(t)))
        self.ctx.synchronize()  # the trace is written on the library's stream
        steps = device_tensor(int(t.value), (r.iterations_completed, 4, r.batch)).cpu().numpy() \
            if r.iterations_completed else np.zeros((0, 4, r.batch), np.float32)
        res = PlanDeviceResult(r.first_action or 0, r.sequence or 0, r.scores or 0, r.best_indices or 0, r.batch,
                               r.scores_cols, r.iterations_completed, r.elapsed_ns * 1e-9,
                               bool(r.deadline_reached), _OUTCOME[r.deadline_outcome])
        return res, steps


# ------------------------------------------------------- device building blocks

def lowest_k_device(ctx: Context, scores_ptr: int, batch: int, samples: int, count: int, out_ptr: int) -> None:
    _check(lib.lwm_lowest_k_device(ctx.handle, VP(scores_ptr), batch, samples, count, VP(out_ptr)))


def color_noise_device(ctx: Context, in_ptr: int, out_ptr: int, batch: int, samples: int, horizon: int,
                       action_dim: int, beta: float) -> None:
    _check(lib.lwm_color_noise_device(ctx.handle, VP(in_ptr), VP(out_ptr), batch, samples, horizon, action_dim,
                                      F(beta)))


def normal_device(ctx: Context, seed: int, offset: int, count: int, out_ptr: int) -> None:
    _check(lib.lwm_normal_device(ctx.handle, U64(seed), U64(offset), C.c_size_t(count), VP(out_ptr)))


# ------------------------------------------------------------ image preprocessing

PACKED_FORMATS = {"rgb": 0, "bgr": 1, "rgba": 2, "bgra": 3}
NV12_COLOR_SPACES = {"bt601-video": 0, "bt709-video": 1, "bt601-full": 2, "bt709-full": 3}


def _ptr(x) -> int:
    return x.data_ptr() if hasattr(x, "data_ptr") else int(x)


def preprocess_packed_device(ctx: Context, frames, batch: int, height: int, width: int, fmt, cfg: ImagePreprocess,
                             out, history_len: int = 0, history_slot: int = 0, bf16: bool = False) -> None:
    """Packed u8 [B,H,W,C] device frames -> normalized NCHW (or a history slot) on the context stream
    (ImagePreprocessor / ImageHistoryPreprocessor, src/media/mod.rs:275-343, 470-543)."""
    f = PACKED_FORMATS[fmt] if isinstance(fmt, str) else int(fmt)
    _check(lib.lwm_preprocess_packed_device(ctx.handle, VP(_ptr(frames)), batch, height, width, f, C.byref(cfg),
                                            history_len, history_slot, int(bf16), VP(_ptr(out))))


def preprocess_packed_patches_device(ctx: Context, frames, batch: int, height: int, width: int, fmt,
                                     cfg: ImagePreprocess, patch: int, out, bf16: bool = False) -> None:
    """Packed frames -> the ViT patch matrix [B, (oh/p)(ow/p), 3 p p] (the NCHW values, permuted)."""
    f = PACKED_FORMATS[fmt] if isinstance(fmt, str) else int(fmt)
    _check(lib.lwm_preprocess_packed_patches_device(ctx.handle, VP(_ptr(frames)), batch, height, width, f,
                                                    C.byref(cfg), patch, int(bf16), VP(_ptr(out))))


def preprocess_nv12_patches_device(ctx: Context, y_plane, uv_plane, batch: int, height: int, width: int, color_space,
                                   cfg: ImagePreprocess, patch: int, out, bf16: bool = False) -> None:
    """NV12 planes -> the ViT patch matrix [B, (oh/p)(ow/p), 3 p p] (the NCHW values, permuted)."""
    cs = NV12_COLOR_SPACES[color_space] if isinstance(color_space, str) else int(color_space)
    _check(lib.lwm_preprocess_nv12_patches_device(ctx.handle, VP(_ptr(y_plane)), VP(_ptr(uv_plane)), batch, height,
                                                  width, cs, C.byref(cfg), patch, int(bf16), VP(_ptr(out))))


def preprocess_nv12_device(ctx: Context, y_plane, uv_plane, batch: int, height: int, width: int, color_space,
                           cfg: ImagePreprocess, out, history_len: int = 0, history_slot: int = 0,
                           bf16: bool = False) -> None:
    """NV12 device planes -> normalized NCHW (or a history slot) on the context stream
    (Nv12Preprocessor / Nv12HistoryPreprocessor, src/media/mod.rs:196-273, 345-468)."""
    cs = NV12_COLOR_SPACES[color_space] if isinstance(color_space, str) else int(color_space)
    _check(lib.lwm_preprocess_nv12_device(ctx.handle, VP(_ptr(y_plane)), VP(_ptr(uv_plane)), batch, height, width,
                                          cs, C.byref(cfg), history_len, history_slot, int(bf16), VP(_ptr(out))))


# --------------------------------------------------------------- fleet loop

def fleet_control_step_device(ctx: Context, step: FleetStep) -> None:
    """commit_observation + reference window + geometric prior of every vehicle, on the device."""
    _check(lib.lwm_fleet_control_step_device(ctx.handle, C.byref(step)))


def plant_step_device(ctx: Context, domains_ptr: int, states_ptr: int, motors_ptr: int, commands_ptr: int,
                      command_stride: int, batch: int, dt: float, substeps: int) -> None:
    """SkyJepaRotorPlant::step x substeps for every vehicle, on the device."""
    _check(lib.lwm_rotor_plant_step_device(ctx.handle, VP(domains_ptr), VP(states_ptr), VP(motors_ptr),
                                           VP(commands_ptr), command_stride, batch, F(dt), substeps))


# ------------------------------------------------------------ control session

WARM_STARTS = {"fresh_prior": 0, "shifted_residual": 1}
DYNAMICS = {"learned": 0, "nominal_physics": 1}


class SessionConfig(C.Structure):
    """SkyJepaSessionConfig + SkyJepaControlConfig (session.rs:40-87, control.rs:72-94)."""
    _fields_ = [("samples", U32), ("horizon", U32), ("planner_seed", U64), ("warm_start", I32),
                ("residual_limit_n", F), ("dynamics", I32), ("trim_multiplier", F), ("dt", F), ("iterations", U32),
                ("temperature", F), ("action_noise", F * 4), ("cost", TrackingCost)]

    @staticmethod
    def paper() -> "SessionConfig":
        c = SessionConfig()
        lib.lwm_skyjepa_session_config_paper(C.byref(c))
        return c


class _ControllerPlan(C.Structure):
    _fields_ = [("action", F * 4), ("prior_action", F * 4), ("action_correction", F * 4), ("action_sequence", FP),
                ("predicted_states", FP), ("best_candidate_score", F), ("plan_ms", C.c_double),
                ("deadline_reached", I32)]


@dataclass
class ControllerPlan:
    """SkyJepaControllerPlan (session.rs:89-100)."""
    action: np.ndarray
    prior_action: np.ndarray
    action_correction: np.ndarray
    action_sequence: np.ndarray
    predicted_states: np.ndarray
    best_candidate_score: float
    plan_ms: float
    deadline_reached: bool


class SkyJepaSession:
    """SkyJepaControllerSession (src/models/skyjepa/session.rs:110-470)."""

    def __init__(self, ctx: Context, config: SessionConfig, initial_state, model: Optional[SkyJepaConfig] = None,
                 weights=None, state_mean=None, state_std=None, action_mean=None, action_std=None):
        self.ctx = ctx
        self.config = config
        w = None if weights is None else _f32(weights)
        h = VP()
        _check(lib.lwm_skyjepa_session_create(
            ctx.handle, C.byref(config), C.byref(model) if model is not None else None, _fp(w),
            C.c_size_t(0 if w is None else w.size), _fp(None if state_mean is None else _f32(state_mean)),
            _fp(None if state_std is None else _f32(state_std)), _fp(None if action_mean is None else _f32(action_mean)),
            _fp(None if action_std is None else _f32(action_std)), _fp(_f32(initial_state)), C.byref(h)))
        self.handle = h
        _LIVE["scorer"].add(self)

    def reset(self, state) -> None:
        _check(lib.lwm_skyjepa_session_reset(self.handle, _fp(_f32(state))))

    def reset_with_action(self, state, action) -> None:
        _check(lib.lwm_skyjepa_session_reset_with_action(self.handle, _fp(_f32(state)), _fp(_f32(action))))

    def commit_observation(self, state, action) -> None:
        _check(lib.lwm_skyjepa_session_commit_observation(self.handle, _fp(_f32(state)), _fp(_f32(action))))

    def plan(self, reference_states, include_prediction: bool = False) -> ControllerPlan:
        T = self.config.horizon
        refs = _f32(reference_states, (T, 18))
        seq = np.empty((T, 4), np.float32)
        pred = np.empty((T, 18), np.float32) if include_prediction else np.empty((0, 18), np.float32)
        r = _ControllerPlan()
        r.action_sequence = _fp(seq)
        r.predicted_states = _fp(pred) if include_prediction else None
        _check(lib.lwm_skyjepa_session_plan(self.handle, _fp(refs), int(include_prediction), C.byref(r)))
        return ControllerPlan(np.array(r.action[:], np.float32), np.array(r.prior_action[:], np.float32),
                              np.array(r.action_correction[:], np.float32), seq, pred, float(r.best_candidate_score),
                              float(r.plan_ms), bool(r.deadline_reached))

    def set_precision(self, precision: str) -> None:
        """Precision of the learned scorer (lwm_scorer_skyjepa_set_precision)."""
        _check(lib.lwm_scorer_skyjepa_set_precision(lib.lwm_skyjepa_session_scorer(self.handle), PRECISIONS[precision]))

    @property
    def trim_scale(self) -> float:
        return float(lib.lwm_skyjepa_session_trim_scale(self.handle))

    def close(self) -> None:
        if getattr(self, "handle", None):
            if getattr(self.ctx, "handle", None):
                lib.lwm_skyjepa_session_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def shifted_residual(sequence, prior, limit: float) -> np.ndarray:
    """shifted_residual (src/models/skyjepa/session.rs:534-543) for one [T, A] sequence."""
    seq = _f32(sequence)
    T, A = seq.shape
    out = np.empty((T, A), np.float32)
    _check(lib.lwm_skyjepa_shifted_residual(_fp(seq), _fp(_f32(prior, (T, A))), T, A, F(limit), _fp(out)))
    return out


# ----------------------------------------------------------------- task inputs

REFERENCE_KINDS = {"hover": 0, "circle": 1, "figure-eight": 2, "figure8": 2}


def reference_horizon(kind: str, time: float, dt: float, horizon: int, radius: float, period: float) -> np.ndarray:
    """skyjepa_reference_horizon (src/skyjepa_task.rs:44-55)."""
    out = np.empty((horizon, 18), np.float32)
    _check(lib.lwm_skyjepa_reference_horizon(REFERENCE_KINDS[kind], F(time), F(dt), horizon, F(radius), F(period),
                                             _fp(out)))
    return out


def geometric_prior(current_state, references, dt: float, domain: Optional[Domain] = None) -> np.ndarray:
    """skyjepa_geometric_action_prior (src/skyjepa_task.rs:118-162)."""
    refs = _f32(references)
    out = np.empty((refs.shape[0], 4), np.float32)
    d = domain or Domain.default()
    _check(lib.lwm_skyjepa_geometric_prior(_fp(_f32(current_state)), _fp(refs), refs.shape[0], F(dt), C.byref(d),
                                           _fp(out)))
    return out


def plant_step(domain: Domain, state: np.ndarray, motors: np.ndarray, command, dt: float) -> None:
    """SkyJepaRotorPlant::step (src/skyjepa_sim.rs:206-270), in place."""
    _check(lib.lwm_rotor_plant_step(C.byref(domain), _fp(state), _fp(motors), _fp(_f32(command)), F(dt)))


def hover_state() -> np.ndarray:
    """SkyJepaRotorState::hover().as_state18() (src/skyjepa_sim.rs:134-154)."""
    s = np.zeros(18, np.float32)
    s[2] = 1.0
    s[6] = s[10] = s[14] = 1.0
    return s

