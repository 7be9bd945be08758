"""Shared helpers of the GPU parity tests."""
import os

import numpy as np

import oracle as O

O.set_threads(os.cpu_count() or 1)

# Tolerances stated by the north-star contract for f32 paths.
COST_REL = 1e-4
ACTION_ABS = 1e-4


def assert_costs_close(ours, ref, rel=COST_REL, floor=1e-6):
    ours, ref = np.asarray(ours, np.float64), np.asarray(ref, np.float64)
    assert ours.shape == ref.shape, (ours.shape, ref.shape)
    err = np.abs(ours - ref)
    bound = rel * np.abs(ref) + floor
    worst = np.argmax(err - bound)
    assert (err <= bound).all(), f"cost mismatch at {np.unravel_index(worst, err.shape)}: {ours.flat[worst]} vs {ref.flat[worst]}"


def assert_actions_close(ours, ref, tol=ACTION_ABS):
    err = np.abs(np.asarray(ours, np.float64) - np.asarray(ref, np.float64))
    assert err.max() <= tol, f"action mismatch {err.max()}"


def assert_same_argmin(best_ours, best_ref, scores_ref, rel=COST_REL, floor=1e-6):
    """Best indices agree, or differ only between scores tied within tolerance."""
    for b, (i, j) in enumerate(zip(best_ours, best_ref)):
        if i != j:
            si, sj = scores_ref[b][i], scores_ref[b][j]
            assert abs(si - sj) <= rel * abs(sj) + floor, (b, i, j, si, sj)


def normals(seed, shape, offset=0):
    return O.normals(seed, offset, int(np.prod(shape))).reshape(shape)


def torch_ptr(t):
    return int(t.data_ptr())
