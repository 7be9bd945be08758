"""Seeded synthetic inputs of the benchmark workloads (no datasets, no
checkpoints: random-init weights and generated trajectories).

nominal(...)  — one-vehicle nominal-physics MPPI: 512 candidates x 15 steps,
                dt 0.05 s, 10 rotor substeps, sigma = 0.15 x hover thrust,
                bounds [0, 2 x hover], temperature 1, figure-eight reference.
skyjepa(...)  — the same vehicle context for learned SkyJEPA MPPI: a 10-step
                state history and 9-step action history at hover trim, seeded
                normalisation statistics and seeded random model weights.
fleet(...)    — many vehicles, each with its own sampled physical parameters.

Every generator is deterministic in its seed.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional

import numpy as np

from . import (ActionBounds, Domain, MppiConfig, SkyJepaConfig, TrackingCost, geometric_prior, hover_state,
               plant_step, reference_horizon)


def rotvec_to_matrix(v: np.ndarray) -> np.ndarray:
    """mat3_from_rotvec (src/data/drone_racing.rs:901-921), row-major 3x3."""
    v = np.asarray(v, dtype=np.float64)
    theta = float(np.linalg.norm(v))
    if theta < 1e-6:
        return np.array([[1.0, -v[2], v[1]], [v[2], 1.0, -v[0]], [-v[1], v[0], 1.0]], dtype=np.float32)
    x, y, z = v / theta
    c, s = math.cos(theta), math.sin(theta)
    oc = 1.0 - c
    return np.array([[c + x * x * oc, x * y * oc - z * s, x * z * oc + y * s],
                     [y * x * oc + z * s, c + y * y * oc, y * z * oc - x * s],
                     [z * x * oc - y * s, z * y * oc + x * s, c + z * z * oc]], dtype=np.float32)


def random_initial_state(rng: np.random.Generator) -> np.ndarray:
    """Hover at z = 1 m, perturbed by U(-0.2, 0.2) m per axis and a
    U(-0.1, 0.1) rad rotation vector."""
    s = hover_state()
    s[0:3] += rng.uniform(-0.2, 0.2, 3).astype(np.float32)
    s[6:15] = rotvec_to_matrix(rng.uniform(-0.1, 0.1, 3)).reshape(-1)
    return s


def tracking_cost_position_velocity() -> TrackingCost:
    """Position / velocity tracking plus control effort (attitude and body
    rate weights off), the nominal-physics workload's cost."""
    return TrackingCost.make(400.0, 40.0, 0.0, 0.0, [0.01, 0.05, 0.05, 0.10])


@dataclass
class NominalWorkload:
    batch: int
    samples: int
    horizon: int
    dt: float
    substeps: int
    trim: float
    hover: float
    initial: np.ndarray          # [B,18]
    motors: np.ndarray           # [B,4]
    reference_states: np.ndarray  # [B,T,18]
    reference_actions: np.ndarray  # [B,T,4]
    warm_start: np.ndarray       # [B,T,4]
    cost: TrackingCost
    mppi: MppiConfig
    domains: Optional[List[Domain]] = None
    t0: float = 0.0


def nominal(seed: int = 0, batch: int = 1, samples: int = 512, horizon: int = 15, dt: float = 0.05,
            substeps: int = 10, iterations: int = 1, cost: Optional[TrackingCost] = None) -> NominalWorkload:
    rng = np.random.default_rng(seed)
    dom = Domain.default()
    hover = dom.hover_force()
    initial = np.stack([random_initial_state(rng) for _ in range(batch)])
    t0 = float(rng.uniform(0.0, 8.0))
    refs = np.stack([reference_horizon("figure-eight", t0, dt, horizon, 2.0, 8.0) for _ in range(batch)])
    motors = np.full((batch, 4), hover, np.float32)
    ref_actions = np.full((batch, horizon, 4), hover, np.float32)
    warm = np.full((batch, horizon, 4), hover, np.float32)
    cfg = MppiConfig(horizon=horizon, samples=samples, action_dim=4, iterations=iterations,
                     action_bounds=ActionBounds.scalar(4, 0.0, 2.0 * hover),
                     noise_std_per_action=[0.15 * hover] * 4, temperature=1.0, seed=seed + 1)
    return NominalWorkload(batch, samples, horizon, dt, substeps, 1.0, hover, initial, motors, refs, ref_actions,
                           warm, cost or tracking_cost_position_velocity(), cfg, None, t0)


@dataclass
class SkyJepaWorkload(NominalWorkload):
    model: Optional[SkyJepaConfig] = None
    weights: Optional[np.ndarray] = None
    state_history: Optional[np.ndarray] = None   # [B,H,18]
    action_history: Optional[np.ndarray] = None  # [B,H-1,4]
    state_mean: Optional[np.ndarray] = None
    state_std: Optional[np.ndarray] = None
    action_mean: Optional[np.ndarray] = None
    action_std: Optional[np.ndarray] = None


def skyjepa(seed: int = 0, batch: int = 1, samples: int = 512, horizon: int = 15, dt: float = 0.05,
            config: Optional[SkyJepaConfig] = None, iterations: int = 1,
            cost: Optional[TrackingCost] = None) -> SkyJepaWorkload:
    base = nominal(seed, batch, samples, horizon, dt, 10, iterations, cost or TrackingCost.paper())
    cfg = config or SkyJepaConfig.wide()
    rng = np.random.default_rng(seed + 1000)
    Hs = cfg.history_steps
    dom = Domain.default()
    hist = np.empty((batch, Hs, 18), np.float32)
    for b in range(batch):
        # history: Hs plant steps at hover trim ending in the initial state
        x = base.initial[b].copy()
        m = np.full(4, base.hover, np.float32)
        states = [x.copy()]
        for _ in range(Hs - 1):
            for _ in range(10):
                plant_step(dom, x, m, np.full(4, base.hover, np.float32), dt / 10)
            states.append(x.copy())
        hist[b] = np.stack(states)
    base.initial = hist[:, -1].copy()
    act_hist = np.full((batch, Hs - 1, 4), base.hover, np.float32)
    w = SkyJepaWorkload(**base.__dict__)
    w.model = cfg
    w.weights = cfg.random_weights(seed + 2000)
    w.state_history = hist
    w.action_history = act_hist
    w.state_mean = (rng.standard_normal(18) * 0.1).astype(np.float32)
    w.state_std = rng.uniform(0.5, 2.0, 18).astype(np.float32)
    w.action_mean = (rng.standard_normal(4) * 0.1 + base.hover).astype(np.float32)
    w.action_std = rng.uniform(0.5, 2.0, 4).astype(np.float32)
    return w


def fleet_domains(seed: int, vehicles: int) -> List[Domain]:
    """Per-vehicle physical parameters: mass x U(0.8, 1.2), arm length x
    U(0.85, 1.15), motor time constant x U(0.7, 1.3) around the nominal."""
    rng = np.random.default_rng(seed + 3000)
    out = []
    for _ in range(vehicles):
        d = Domain.default()
        d.mass = float(np.float32(d.mass * rng.uniform(0.8, 1.2)))
        d.arm_length = float(np.float32(d.arm_length * rng.uniform(0.85, 1.15)))
        d.motor_time_constant = float(np.float32(d.motor_time_constant * rng.uniform(0.7, 1.3)))
        out.append(d)
    return out


def prior_warm_start(w: NominalWorkload) -> np.ndarray:
    """Geometric prior of every vehicle (the session's warm start)."""
    return np.stack([geometric_prior(w.initial[b], w.reference_states[b], w.dt) for b in range(w.batch)])


def fleet(seed: int = 0, vehicles: int = 256, samples: int = 4096, horizon: int = 30, dt: float = 0.05,
          config: Optional[SkyJepaConfig] = None) -> SkyJepaWorkload:
    """Fleet-scale learned MPPI: `vehicles` independent vehicles with sampled
    physical parameters (fleet_domains), each planning `samples` candidates x
    `horizon` steps with the learned SkyJEPA scorer.  Each vehicle's history
    is flown at its own hover thrust; `masses` carries the per-vehicle mass
    for the scorer's rotor-forces integrator."""
    w = skyjepa(seed, batch=vehicles, samples=samples, horizon=horizon, dt=dt, config=config)
    doms = fleet_domains(seed, vehicles)
    Hs = w.model.history_steps
    for b, d in enumerate(doms):
        hover = d.hover_force()
        x = w.state_history[b, 0].copy()
        states = [x.copy()]
        m = np.full(4, hover, np.float32)
        for _ in range(Hs - 1):
            for _ in range(10):
                plant_step(d, x, m, np.full(4, hover, np.float32), dt / 10)
            states.append(x.copy())
        w.state_history[b] = np.stack(states)
        w.action_history[b] = hover
    w.initial = w.state_history[:, -1].copy()
    w.masses = np.array([d.mass for d in doms], np.float32)
    w.domains = doms
    return w


@dataclass
class LewmWorkload:
    config: object            # LewmConfig
    weights: np.ndarray
    batch: int
    samples: int
    horizon: int
    planner: object           # CemConfig or MppiConfig
    obs: Optional[np.ndarray] = None        # vector observations [B, obs_dim]
    goal_obs: Optional[np.ndarray] = None
    y_plane: Optional[np.ndarray] = None    # NV12 observation / goal frames [B, H, W], [B, H/2, W/2, 2]
    uv_plane: Optional[np.ndarray] = None
    goal_y: Optional[np.ndarray] = None
    goal_uv: Optional[np.ndarray] = None


def lewm_vector(seed: int = 0, batch: int = 1, samples: int = 300, horizon: int = 5, elites: int = 30,
                iterations: int = 3, config=None) -> LewmWorkload:
    """Vector-observation LeWM CEM: 16-d observation and goal ~ N(0, 1),
    300 candidates x 5 steps, 30 elites, 3 iterations, initial std 1 in a
    [-1, 1] box, action dim 2."""
    from . import ActionBounds, CemConfig, LewmConfig
    cfg = config or LewmConfig.vector()
    rng = np.random.default_rng(seed + 4000)
    obs = rng.standard_normal((batch, cfg.obs_dim)).astype(np.float32)
    goal = rng.standard_normal((batch, cfg.obs_dim)).astype(np.float32)
    cem = CemConfig(horizon=horizon, samples=samples, elites=elites, action_dim=cfg.action_dim,
                    iterations=iterations, action_bounds=ActionBounds.symmetric(cfg.action_dim, 1.0), init_std=1.0,
                    min_std=1e-3, seed=seed + 1)
    return LewmWorkload(cfg, cfg.random_weights(seed + 5000), batch, samples, horizon, cem, obs=obs, goal_obs=goal)


def lewm_image(seed: int = 0, batch: int = 1, samples: int = 1024, horizon: int = 10, config=None) -> LewmWorkload:
    """Image LeWM MPPI: seeded uniform-noise NV12 observation and goal frames
    at the model's image size, 1024 candidates x 10 steps, action dim 2,
    temperature 0.5, std 1 in a [-1, 1] box."""
    from . import ActionBounds, LewmConfig, MppiConfig
    cfg = config or LewmConfig.image()
    rng = np.random.default_rng(seed + 6000)
    s = cfg.image_size
    planes = [rng.integers(0, 256, shape, dtype=np.uint8)
              for shape in ((batch, s, s), (batch, s // 2, s // 2, 2), (batch, s, s), (batch, s // 2, s // 2, 2))]
    mppi = MppiConfig(horizon=horizon, samples=samples, action_dim=cfg.action_dim, iterations=1,
                      action_bounds=ActionBounds.symmetric(cfg.action_dim, 1.0), noise_std=1.0, temperature=0.5,
                      seed=seed + 1)
    return LewmWorkload(cfg, cfg.random_weights(seed + 7000), batch, samples, horizon, mppi, y_plane=planes[0],
                        uv_plane=planes[1], goal_y=planes[2], goal_uv=planes[3])
