"""The allocation-free nominal MPPI iteration (lwm_nominal_mppi_noalloc).

Callers that cannot allocate device memory once they run (real-time control
loops, runtimes that reserve all memory at start-up) use this entry point with
their own buffers; its scratch is a static array inside the library.  These
tests call it through the C ABI and check it against the planner path
(lwm_plan with an MPPI planner and the nominal scorer) on two iterations in a
row, the second fed with the first's warm start — with injected noise and
with the Philox draws of a seeded planner, on the default stream and on a
stream the caller created, at the default horizon and at horizon 64 — and
check that oversized requests are refused without GPU work.  This file is
collected last.
"""
import ctypes as C

import numpy as np
import pytest

import lewm_b200 as L
from gpu_helpers import assert_actions_close, assert_costs_close, normals
from lewm_b200 import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

FP = C.c_void_p


class NominalMppiIo(C.Structure):
    _fields_ = [("initial", FP), ("motors", FP), ("reference_states", FP), ("reference_actions", FP),
                ("domains", FP), ("mean", FP), ("std", FP), ("injected_noise", FP), ("scores", FP),
                ("sequence", FP), ("first_action", FP), ("warm_start", FP), ("best_indices", FP)]


fn = L.lib.lwm_nominal_mppi_noalloc
fn.restype = C.c_int
fn.argtypes = [C.c_int, C.c_void_p, C.POINTER(L.NominalScorerConfig), C.c_uint32, C.c_uint32, C.c_uint32,
               C.POINTER(C.c_float), C.POINTER(C.c_float), C.c_float, C.c_uint64, C.c_uint64,
               C.POINTER(NominalMppiIo)]


def _call(cfg, B, S, T, low, high, temperature, io, stream=None, seed=0, offset=0):
    lo = (C.c_float * 4)(*low)
    hi = (C.c_float * 4)(*high)
    return fn(0, stream, C.byref(cfg), B, S, T, lo, hi, temperature, seed, offset, C.byref(io))


def _dev(a):
    return torch.as_tensor(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def _run_both(ctx, batch, samples, horizon, philox, side_stream):
    """Two iterations in a row on the planner path (lwm_plan, MPPI planner and
    nominal scorer) and on the allocation-free entry point, the second fed
    with the first one's warm start; noise injected, or Philox draws from the
    planner's seed at the offsets its draw reservation gives each plan."""
    w = W.nominal(seed=7, batch=batch, samples=samples, horizon=horizon)
    B, S, T = w.batch, w.samples, w.horizon
    hover = w.hover
    low, high = [0.0] * 4, [2.0 * hover] * 4
    seed = 4242
    noise = None if philox else [normals(500 + i, (B, S, T, 4)) for i in range(2)]
    if philox:
        w.mppi.seed = seed

    # the planner path
    planner = L.MppiPlanner(ctx, w.mppi)
    planner.set_warm_start_sequence(w.warm_start)
    scorer = L.NominalScorer(ctx, w.dt, w.trim, w.cost, w.substeps)
    scorer.set_context(w.initial, w.motors, w.reference_states, w.reference_actions)
    ref = [planner.plan(scorer, injected_noise=None if philox else noise[i][None]) for i in range(2)]
    per_plan = B * S * T * 4 + (B * S * T * 4) % 2   # round_even(B*S*T*A) draws per plan

    # the allocation-free path on caller-owned buffers
    cfg = L.NominalScorerConfig(w.dt, w.trim, w.substeps, w.cost, L.Domain.default())
    domains = np.frombuffer(bytes((L.Domain * B)(*([L.Domain.default()] * B))), dtype=np.float32).copy()
    std = np.full((B, T, 4), 0.15 * hover, np.float32)
    bufs = {"initial": _dev(w.initial), "motors": _dev(w.motors), "reference_states": _dev(w.reference_states),
            "reference_actions": _dev(w.reference_actions), "domains": _dev(domains), "std": _dev(std)}
    mean = _dev(w.warm_start)
    stream = torch.cuda.Stream() if side_stream else None
    torch.cuda.synchronize()
    for i in range(2):
        out = {"scores": torch.full((B, S), float("nan"), device="cuda"),
               "sequence": torch.full((B, T, 4), float("nan"), device="cuda"),
               "first_action": torch.full((B, 4), float("nan"), device="cuda"),
               "warm_start": torch.full((B, T, 4), float("nan"), device="cuda"),
               "best_indices": torch.full((B,), -1, dtype=torch.int32, device="cuda")}
        nz = None if philox else _dev(noise[i])
        io = NominalMppiIo(*(b.data_ptr() for b in (bufs["initial"], bufs["motors"], bufs["reference_states"],
                                                   bufs["reference_actions"], bufs["domains"])),
                           mean.data_ptr(), bufs["std"].data_ptr(), None if nz is None else nz.data_ptr(),
                           *(out[k].data_ptr() for k in ("scores", "sequence", "first_action", "warm_start",
                                                         "best_indices")))
        torch.cuda.synchronize()
        status = _call(cfg, B, S, T, low, high, w.mppi.temperature, io,
                       stream=None if stream is None else stream.cuda_stream, seed=seed, offset=i * per_plan)
        assert status == 0, L.lib.lwm_last_error().decode()
        if stream is not None:
            stream.synchronize()
        torch.cuda.synchronize()
        assert torch.cuda.current_device() == 0
        assert_costs_close(out["scores"].cpu().numpy(), ref[i].scores)
        assert_actions_close(out["sequence"].cpu().numpy(), ref[i].sequence)
        assert_actions_close(out["first_action"].cpu().numpy(), ref[i].first_action)
        assert out["best_indices"].cpu().numpy().astype(np.uint32).tolist() == ref[i].best_indices
        mean = out["warm_start"]  # the next iteration starts from the shifted sequence
    assert_actions_close(mean.cpu().numpy(), planner.warm_start_sequence())
    planner.close()
    scorer.close()


def test_noalloc_iteration_matches_planner_on_two_calls(ctx):
    _run_both(ctx, batch=2, samples=200, horizon=15, philox=False, side_stream=False)


def test_noalloc_philox_draws_match_seeded_planner(ctx):
    # injected_noise NULL: the kernel draws Philox normals from (seed, offset)
    _run_both(ctx, batch=2, samples=200, horizon=15, philox=True, side_stream=False)


def test_noalloc_long_horizon_on_caller_stream(ctx):
    # horizon 64 needs more than 48 KB of dynamic shared memory per block;
    # the work runs on a stream the caller created
    _run_both(ctx, batch=1, samples=512, horizon=64, philox=False, side_stream=True)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    dummy = torch.zeros(16, device="cuda")
    p = dummy.data_ptr()
    io = NominalMppiIo(*([p] * 13))
    cfg = L.NominalScorerConfig(0.05, 1.0, 10, L.TrackingCost.paper(), L.Domain.default())
    status = _call(cfg, 2000, 64, 15, [0.0] * 4, [6.0] * 4, 1.0, io)
    assert status == 1 and "exceeds the no-alloc limit of 1024 vehicles" in L.lib.lwm_last_error().decode()
    status = _call(cfg, 256, 4096, 30, [0.0] * 4, [6.0] * 4, 1.0, io)
    assert status == 1 and "the no-alloc limit is" in L.lib.lwm_last_error().decode()
    torch.cuda.synchronize()
