"""Candidate shards of CEM / iCEM plans (lwm_planner_set_shard_exchange)
against the same plan unsharded: each shard reduces its candidates to its
lowest `elites`, the shards exchange those tuples every iteration, and every
shard refits from the merged set, so the sharded plan is the unsharded one
bit for bit (same Philox draws, same elites in the same order).

The shards run here as threads on one GPU, each with its own context; the
exchange is a host-side all-gather between the threads (the NCCL exchange of
lewm_b200.fleet.nccl_elite_exchange runs in the two-GPU tests)."""
import threading

import numpy as np
import pytest

import lewm_b200 as L
from lewm_b200 import fleet as F
from lewm_b200 import workloads as W

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


class ThreadExchange:
    """All-gather of device buffers between shard threads (staged on the host)."""

    def __init__(self, shards):
        self.shards = shards
        self.parts = [None] * shards
        self.barrier = threading.Barrier(shards, timeout=60)

    def for_rank(self, rank, ctx):
        def exchange(local_ptr, count, gathered_ptr, _stream):
            with torch.cuda.stream(ctx.torch_stream()):
                self.parts[rank] = L.device_tensor(local_ptr, (count,)).cpu()  # synchronises the stream
            self.barrier.wait()
            full = torch.cat(self.parts)
            with torch.cuda.stream(ctx.torch_stream()):
                L.device_tensor(gathered_ptr, (self.shards * count,)).copy_(full)
                torch.cuda.current_stream().synchronize()
            self.barrier.wait()  # every rank has read the parts before the next iteration writes them
        return exchange


def _nominal_scorer(ctx, w):
    sc = L.NominalScorer(ctx, w.dt, w.trim, w.cost, w.substeps)
    sc.set_context(w.initial, w.motors, w.reference_states, w.reference_actions)
    return sc


def _plan_sharded(make_planner, make_scorer, S, bounds, warm=None):
    shards = len(bounds)
    ex = ThreadExchange(shards)
    out = [None] * shards
    errors = []

    def run(rank):
        try:
            ctx = L.Context(0)
            s0, s1 = bounds[rank]
            p = make_planner(ctx, s1 - s0)
            p.set_shard(s0, S)
            p.set_shard_exchange(shards, ex.for_rank(rank, ctx))
            if warm is not None:
                p.set_warm_start_sequence(warm)
            sc = make_scorer(ctx)
            r = p.plan(sc)
            out[rank] = (r, p.warm_start_sequence() if warm is not None else None)
            p.close()
            sc.close()
            ctx.close()
        except Exception as e:  # noqa: BLE001 - surfaced below
            errors.append(e)
            ex.barrier.abort()

    threads = [threading.Thread(target=run, args=(k,)) for k in range(shards)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(120)
    assert not errors, errors
    return out


@pytest.mark.parametrize("kind", ["cem", "icem"])
@pytest.mark.parametrize("bounds", [[(0, 128), (128, 256)], [(0, 100), (100, 170), (170, 256)]])
def test_elite_shards_equal_unsharded(ctx, kind, bounds):
    w = W.nominal(seed=21, batch=2, samples=256, horizon=10)
    hover = w.hover
    if kind == "cem":
        cfg = L.CemConfig(horizon=10, samples=256, elites=24, action_dim=4, iterations=3,
                          action_bounds=L.ActionBounds.scalar(4, 0.0, 2 * hover), init_std=0.6 * hover, seed=9)
        make = lambda c, S: L.CemPlanner(c, _resize(cfg, S))
        warm = None
    else:
        cfg = L.IcemConfig(horizon=10, samples=256, elites=24, action_dim=4, keep_elites=5, iterations=3,
                           noise_beta=2.0, alpha=0.1, init_std=0.6 * hover,
                           action_bounds=L.ActionBounds.scalar(4, 0.0, 2 * hover), seed=9)
        make = lambda c, S: L.IcemPlanner(c, _resize(cfg, S))
        warm = w.warm_start
    full = make(ctx, 256)
    if warm is not None:
        full.set_warm_start_sequence(warm)
    ref = full.plan(_nominal_scorer(ctx, w))
    ref_warm = full.warm_start_sequence() if warm is not None else None
    got = _plan_sharded(make, lambda c: _nominal_scorer(c, w), 256, bounds, warm)
    for rank, (r, wr) in enumerate(got):
        s0, s1 = bounds[rank]
        assert np.array_equal(r.sequence, ref.sequence)
        assert np.array_equal(r.first_action, ref.first_action)
        assert r.best_indices == ref.best_indices
        assert np.array_equal(r.scores, ref.scores[:, s0:s1])
        if wr is not None:
            assert np.array_equal(wr, ref_warm)


def _resize(cfg, samples):
    import dataclasses
    return dataclasses.replace(cfg, samples=samples)


def test_elite_shard_validation(ctx):
    p = L.CemPlanner(ctx, L.CemConfig(horizon=4, samples=16, elites=8, action_dim=2, iterations=2))
    sc = L.CallbackScorer(ctx, 1, lambda c: (c ** 2).sum(dim=(2, 3)))
    p.set_shard(0, 32)
    with pytest.raises(L.LwmError, match="need an elite exchange"):
        p.plan(sc)
    with pytest.raises(L.LwmError, match="exceed sample_total"):
        p.set_shard(24, 32)
    m = L.MppiPlanner(ctx, L.MppiConfig(horizon=4, samples=16, action_dim=2))
    with pytest.raises(L.LwmError, match="lwm_mppi_combine_device"):
        m.set_shard_exchange(2, lambda *a: None)
    assert F.nccl_elite_exchange  # the NCCL form used by multi-GPU callers
