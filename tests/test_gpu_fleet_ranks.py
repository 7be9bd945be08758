"""Fleet planning over two GPUs (one process per GPU, NCCL) against the same
fleet planned by one process on one GPU.  Vehicle groups must give the
single-GPU result exactly; candidate shards (one all-gather of the per-vehicle
MPPI tuples and the combine kernel) up to the order of the float sums.
A vehicle range draws the noise of a planner over that range alone, so the
reference plan of a rank is its own vehicle range on one GPU.
Skipped unless two GPUs are visible."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

V, S, T = 4, 512, 15


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _scorer(L, ctx, full, sl, precision):
    sc = L.SkyJepaScorer(ctx, full.model, full.weights, full.state_mean, full.state_std, full.action_mean,
                         full.action_std, full.cost, full.dt)
    sc.set_precision(precision)
    sc.set_context(full.state_history[sl].copy(), full.action_history[sl].copy(), full.reference_states[sl].copy(),
                   full.reference_actions[sl].copy(), vehicle_mass=full.masses[sl].copy())
    return sc


def _plan(L, F, ctx, part, full, precision, group):
    sl = slice(*part.vehicles)
    sc = _scorer(L, ctx, full, sl, precision)
    fp = F.FleetPlanner(ctx, part, sc, full.mppi, group)
    fp.planner.set_warm_start_sequence(full.warm_start[sl])
    seqs = []
    for _ in range(2):  # the second plan starts from the shifted warm start
        res = fp.plan_device()
        ctx.synchronize()
        seqs.append(L.device_tensor(res.sequence, (sl.stop - sl.start, T, 4)).cpu().numpy())
    fp.close()
    sc.close()
    return np.stack(seqs)


def _rank_main(rank, world, port, mode, precision, out_dir):
    import datetime
    import torch.distributed as dist
    import lewm_b200 as L
    from lewm_b200 import fleet as F
    from lewm_b200 import workloads as W
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method="env://", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        parts = F.partition(V, S, world, mode)
        group = F.new_groups(parts)
        full = W.fleet(seed=12, vehicles=V, samples=S, horizon=T)
        ctx = L.Context(rank)
        seq = _plan(L, F, ctx, parts[rank], full, precision, group)
        np.save(os.path.join(out_dir, f"rank{rank}.npy"), seq)
        ctx.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("mode", ["vehicles", "candidates"])
@pytest.mark.parametrize("precision", ["f32", "bf16"])
def test_two_gpu_fleet_equals_one_gpu(tmp_path, mode, precision):
    import torch.multiprocessing as mp
    import lewm_b200 as L
    from lewm_b200 import fleet as F
    from lewm_b200 import workloads as W
    mp.start_processes(_rank_main, args=(2, _free_port(), mode, precision, str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    import dataclasses
    full = W.fleet(seed=12, vehicles=V, samples=S, horizon=T)
    ctx = L.Context(0)
    whole = F.partition(V, S, 1)[0]
    for p in F.partition(V, S, 2, mode):
        # the same vehicle range planned by one process over all S candidates
        want = _plan(L, F, ctx, dataclasses.replace(whole, vehicles=p.vehicles), full, precision, None)
        got = np.load(tmp_path / f"rank{p.rank}.npy")
        if mode == "vehicles":
            assert np.array_equal(got, want)
        else:
            # the MPPI-weighted mean of the same candidates, summed in another order
            np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-4 * float(np.abs(want).max()))
    ctx.close()


def _elite_rank_main(rank, world, port, kind, out_dir):
    import dataclasses
    import datetime
    import torch.distributed as dist
    import lewm_b200 as L
    from lewm_b200 import fleet as F
    from lewm_b200 import workloads as W
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method="env://", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        w = W.nominal(seed=21, batch=2, samples=256, horizon=10)
        cfg = _elite_cfg(L, kind, w.hover)
        s0, s1 = F.split_range(256, world, rank)
        ctx = L.Context(rank)
        planner = (L.CemPlanner if kind == "cem" else L.IcemPlanner)(ctx, dataclasses.replace(cfg, samples=s1 - s0))
        planner.set_shard(s0, 256)
        planner.set_shard_exchange(world, F.nccl_elite_exchange(ctx, dist.group.WORLD, world))
        if kind == "icem":
            planner.set_warm_start_sequence(w.warm_start)
        sc = L.NominalScorer(ctx, w.dt, w.trim, w.cost, w.substeps)
        sc.set_context(w.initial, w.motors, w.reference_states, w.reference_actions)
        r = planner.plan(sc)
        np.savez(os.path.join(out_dir, f"elite{rank}.npz"), sequence=r.sequence, scores=r.scores,
                 best=np.array(r.best_indices))
        planner.close()
        sc.close()
        ctx.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _elite_cfg(L, kind, hover):
    bounds = L.ActionBounds.scalar(4, 0.0, 2 * hover)
    if kind == "cem":
        return L.CemConfig(horizon=10, samples=256, elites=24, action_dim=4, iterations=3, action_bounds=bounds,
                           init_std=0.6 * hover, seed=9)
    return L.IcemConfig(horizon=10, samples=256, elites=24, action_dim=4, keep_elites=5, iterations=3,
                        noise_beta=2.0, alpha=0.1, init_std=0.6 * hover, action_bounds=bounds, seed=9)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("kind", ["cem", "icem"])
def test_two_gpu_elite_shards_equal_one_gpu(tmp_path, kind):
    # CEM / iCEM candidate shards exchanging elite tuples with one NCCL
    # all-gather per iteration reproduce the unsharded plan bit for bit
    import torch.multiprocessing as mp
    import lewm_b200 as L
    from lewm_b200 import fleet as F
    from lewm_b200 import workloads as W
    mp.start_processes(_elite_rank_main, args=(2, _free_port(), kind, str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    w = W.nominal(seed=21, batch=2, samples=256, horizon=10)
    ctx = L.Context(0)
    planner = (L.CemPlanner if kind == "cem" else L.IcemPlanner)(ctx, _elite_cfg(L, kind, w.hover))
    if kind == "icem":
        planner.set_warm_start_sequence(w.warm_start)
    sc = L.NominalScorer(ctx, w.dt, w.trim, w.cost, w.substeps)
    sc.set_context(w.initial, w.motors, w.reference_states, w.reference_actions)
    ref = planner.plan(sc)
    for rank in range(2):
        s0, s1 = F.split_range(256, 2, rank)
        got = np.load(tmp_path / f"elite{rank}.npz")
        assert np.array_equal(got["sequence"], ref.sequence)
        assert got["best"].tolist() == ref.best_indices
        assert np.array_equal(got["scores"], ref.scores[:, s0:s1])
    planner.close()
    sc.close()
    ctx.close()
