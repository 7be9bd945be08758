"""The CPU reference arm builds its workload from the oracle alone
(oracle/workload.py, no product import); these tests pin it to the
product's own workload generator (lewm_b200.workloads): the same arrays,
weights and configurations for the same seed."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import workload as OW
from lewm_b200 import workloads as W


def _same_struct(a, b):
    assert C.sizeof(a) == C.sizeof(b)
    assert bytes(a) == bytes(b)


@pytest.mark.parametrize("make, kw", [("nominal", dict(seed=17)), ("skyjepa", dict(seed=17)),
                                      ("skyjepa", dict(seed=3, batch=2, samples=256, horizon=7))])
def test_oracle_workload_equals_product_workload(make, kw):
    a = getattr(W, make)(**kw)
    b = getattr(OW, make)(**kw)
    for name in ("initial", "motors", "reference_states", "reference_actions", "warm_start"):
        assert np.array_equal(getattr(a, name), getattr(b, name)), name
    assert (a.hover, a.dt, a.samples, a.horizon, a.batch) == (b.hover, b.dt, b.samples, b.horizon, b.batch)
    _same_struct(a.cost, b.cost)
    _same_struct(a.mppi._c(), b.mppi._c())
    if make == "skyjepa":
        _same_struct(a.model, b.model)
        for name in ("weights", "state_history", "action_history", "state_mean", "state_std", "action_mean",
                     "action_std"):
            assert np.array_equal(getattr(a, name), getattr(b, name)), name


def test_oracle_fleet_workload_equals_product_fleet_workload():
    a = W.fleet(seed=23, vehicles=6, samples=128, horizon=9)
    b = OW.fleet(seed=23, vehicles=6, samples=128, horizon=9)
    for name in ("initial", "state_history", "action_history", "masses", "reference_states", "weights"):
        assert np.array_equal(getattr(a, name), getattr(b, name)), name
    for da, db in zip(a.domains, b.domains):
        _same_struct(da, db)


def test_oracle_defaults_equal_product_defaults():
    import lewm_b200 as L
    _same_struct(L.Domain.default(), O.Domain.default())
    _same_struct(L.TrackingCost.paper(), O.TrackingCost.paper())
    _same_struct(L.SkyJepaConfig.paper(), O.SkyJepaConfig.paper())
    _same_struct(L.SkyJepaConfig.wide(), O.SkyJepaConfig.wide())
    cfg = O.SkyJepaConfig.paper()
    assert np.array_equal(L.SkyJepaConfig.paper().random_weights(5), cfg.random_weights(5))
