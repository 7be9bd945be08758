"""Seeded synthetic inputs of the benchmark's SkyJEPA and nominal workloads,
built from the oracle alone (TEST INFRASTRUCTURE ONLY: the CPU reference arm
of bench.py and the tests use it; it imports nothing from the product).

The same workloads as the product's `lewm_b200.workloads` (nominal, skyjepa,
fleet), value for value: the same numpy generators consumed in the same
order, the reference's default domain / cost / model configuration, the
oracle's plant, reference trajectories and seeded weights.
tests/test_oracle_workload.py checks that both give identical arrays.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import List, Optional, Sequence

import numpy as np

import oracle as O

FIGURE_EIGHT = 2  # skyjepa_reference_state's kind (src/skyjepa_task.rs)


@dataclass
class ActionBounds:
    """ActionBounds (src/planner.rs:67-83)."""
    low: List[float]
    high: List[float]

    @staticmethod
    def scalar(action_dim: int, low: float, high: float) -> "ActionBounds":
        return ActionBounds([low] * action_dim, [high] * action_dim)


@dataclass
class MppiConfig:
    """MppiConfig (src/planner.rs:178-208) as the oracle planner takes it;
    defaults of MppiConfig::new (iterations 1, bounds [-1, 1], noise 1,
    temperature 1, no deadline)."""
    horizon: int
    samples: int
    action_dim: int
    iterations: int = 1
    action_bounds: Optional[ActionBounds] = None
    noise_std: float = 1.0
    noise_std_per_action: Optional[Sequence[float]] = None
    temperature: float = 1.0
    seed: Optional[int] = None

    def _c(self) -> O._MppiConfig:
        c = O._MppiConfig()
        c.horizon, c.samples, c.iterations, c.action_dim = self.horizon, self.samples, self.iterations, self.action_dim
        b = self.action_bounds or ActionBounds.scalar(self.action_dim, -1.0, 1.0)
        for i in range(self.action_dim):
            c.bounds_low[i], c.bounds_high[i] = b.low[i], b.high[i]
        c.noise_std = self.noise_std
        if self.noise_std_per_action is not None:
            c.has_noise_std_per_action = 1
            for i, v in enumerate(self.noise_std_per_action):
                c.noise_std_per_action[i] = v
        c.temperature = self.temperature
        c.deadline_ns = -1
        if self.seed is not None:
            c.has_seed, c.seed = 1, self.seed
        return c


def hover_state() -> np.ndarray:
    """SkyJepaRotorState::hover().as_state18() (src/skyjepa_sim.rs:134-154)."""
    s = np.zeros(18, np.float32)
    s[2] = 1.0
    s[6] = s[10] = s[14] = 1.0
    return s


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
    s = hover_state()
    s[0:3] += rng.uniform(-0.2, 0.2, 3).astype(np.float32)
    s[6:15] = rotvec_to_matrix(rng.uniform(-0.1, 0.1, 3)).reshape(-1)
    return s


@dataclass
class Workload:
    batch: int
    samples: int
    horizon: int
    dt: float
    substeps: int
    trim: float
    hover: float
    initial: np.ndarray
    motors: np.ndarray
    reference_states: np.ndarray
    reference_actions: np.ndarray
    warm_start: np.ndarray
    cost: O.TrackingCost
    mppi: MppiConfig
    domains: Optional[List[O.Domain]] = None
    t0: float = 0.0
    model: Optional[O.SkyJepaConfig] = None
    weights: Optional[np.ndarray] = None
    state_history: Optional[np.ndarray] = None
    action_history: Optional[np.ndarray] = None
    state_mean: Optional[np.ndarray] = None
    state_std: Optional[np.ndarray] = None
    action_mean: Optional[np.ndarray] = None
    action_std: Optional[np.ndarray] = None
    masses: Optional[np.ndarray] = None


def nominal(seed: int = 0, batch: int = 1, samples: int = 512, horizon: int = 15, dt: float = 0.05,
            substeps: int = 10, iterations: int = 1, cost: Optional[O.TrackingCost] = None) -> Workload:
    rng = np.random.default_rng(seed)
    dom = O.Domain.default()
    hover = dom.hover_force()
    initial = np.stack([random_initial_state(rng) for _ in range(batch)])
    t0 = float(rng.uniform(0.0, 8.0))
    refs = np.stack([O.reference_horizon(FIGURE_EIGHT, t0, dt, horizon, 2.0, 8.0) for _ in range(batch)])
    motors = np.full((batch, 4), hover, np.float32)
    ref_actions = np.full((batch, horizon, 4), hover, np.float32)
    warm = np.full((batch, horizon, 4), hover, np.float32)
    cfg = MppiConfig(horizon=horizon, samples=samples, action_dim=4, iterations=iterations,
                     action_bounds=ActionBounds.scalar(4, 0.0, 2.0 * hover),
                     noise_std_per_action=[0.15 * hover] * 4, temperature=1.0, seed=seed + 1)
    cost = cost or O.TrackingCost.make(400.0, 40.0, 0.0, 0.0, [0.01, 0.05, 0.05, 0.10])
    return Workload(batch, samples, horizon, dt, substeps, 1.0, hover, initial, motors, refs, ref_actions, warm,
                    cost, cfg, None, t0)


def skyjepa(seed: int = 0, batch: int = 1, samples: int = 512, horizon: int = 15, dt: float = 0.05,
            iterations: int = 1) -> Workload:
    w = nominal(seed, batch, samples, horizon, dt, 10, iterations, O.TrackingCost.paper())
    cfg = O.SkyJepaConfig.wide()
    rng = np.random.default_rng(seed + 1000)
    Hs = cfg.history_steps
    dom = O.Domain.default()
    hist = np.empty((batch, Hs, 18), np.float32)
    for b in range(batch):
        x = w.initial[b].copy()
        m = np.full(4, w.hover, np.float32)
        states = [x.copy()]
        for _ in range(Hs - 1):
            for _ in range(10):
                O.plant_step(dom, x, m, np.full(4, w.hover, np.float32), dt / 10)
            states.append(x.copy())
        hist[b] = np.stack(states)
    w.initial = hist[:, -1].copy()
    w.model = cfg
    w.weights = cfg.random_weights(seed + 2000)
    w.state_history = hist
    w.action_history = np.full((batch, Hs - 1, 4), w.hover, np.float32)
    w.state_mean = (rng.standard_normal(18) * 0.1).astype(np.float32)
    w.state_std = rng.uniform(0.5, 2.0, 18).astype(np.float32)
    w.action_mean = (rng.standard_normal(4) * 0.1 + w.hover).astype(np.float32)
    w.action_std = rng.uniform(0.5, 2.0, 4).astype(np.float32)
    return w


def fleet_domains(seed: int, vehicles: int) -> List[O.Domain]:
    rng = np.random.default_rng(seed + 3000)
    out = []
    for _ in range(vehicles):
        d = O.Domain.default()
        d.mass = float(np.float32(d.mass * rng.uniform(0.8, 1.2)))
        d.arm_length = float(np.float32(d.arm_length * rng.uniform(0.85, 1.15)))
        d.motor_time_constant = float(np.float32(d.motor_time_constant * rng.uniform(0.7, 1.3)))
        out.append(d)
    return out


def fleet(seed: int = 0, vehicles: int = 256, samples: int = 4096, horizon: int = 30, dt: float = 0.05) -> Workload:
    w = skyjepa(seed, batch=vehicles, samples=samples, horizon=horizon, dt=dt)
    doms = fleet_domains(seed, vehicles)
    Hs = w.model.history_steps
    for b, d in enumerate(doms):
        hover = d.hover_force()
        x = w.state_history[b, 0].copy()
        states = [x.copy()]
        m = np.full(4, hover, np.float32)
        for _ in range(Hs - 1):
            for _ in range(10):
                O.plant_step(d, x, m, np.full(4, hover, np.float32), dt / 10)
            states.append(x.copy())
        w.state_history[b] = np.stack(states)
        w.action_history[b] = hover
    w.initial = w.state_history[:, -1].copy()
    w.masses = np.array([d.mass for d in doms], np.float32)
    w.domains = doms
    return w
