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


def assert_same_elites(ours, ref_elites, ref_iteration_scores, rel=COST_REL, floor=1e-6):
    """Every iteration's elite indices, in selection order (ascending score,
    ties to the lower index), equal the oracle's except where the two
    candidates at a position have scores tied within the cost tolerance (the
    contract's "bit-exact except for ties").  After an iteration whose
    selection differs by such a tie, the next iteration refits from a
    different elite set and is no longer comparable: the check stops there.
    Returns the number of iterations compared exactly."""
    ours = np.asarray(ours)
    ref_elites = np.asarray(ref_elites)
    assert ours.shape == ref_elites.shape, (ours.shape, ref_elites.shape)
    for it in range(ours.shape[0]):
        differs = False
        for b in range(ours.shape[1]):
            o, r = ours[it, b], ref_elites[it, b]
            if np.array_equal(o, r):
                continue
            differs = True
            sc = np.asarray(ref_iteration_scores[it, b], np.float64)
            for j in np.nonzero(o != r)[0]:
                si, sj = sc[o[j]], sc[r[j]]
                assert abs(si - sj) <= rel * abs(sj) + floor, \
                    f"iteration {it}, vehicle {b}, elite {j}: candidate {o[j]} ({si}) vs oracle {r[j]} ({sj})"
        if differs:
            return it
    return ours.shape[0]


def normals(seed, shape, offset=0):
    return O.normals(seed, offset, int(np.prod(shape))).reshape(shape)


def torch_ptr(t):
    return int(t.data_ptr())
