"""Fleet partitioning and the cross-GPU MPPI exchange without a GPU.

The partition and the tuple exchange of lewm_b200.fleet run here as gloo
ranks on CPU (world sizes 2 and 4).  Each rank reduces its candidate range to
per-vehicle MPPI tuples with a numpy restatement of the kernels' tuple math,
the ranks exchange them through fleet.exchange_tuples, and the combined plan
must equal the oracle's unsharded mppi_weighted_sequence
(src/planner.rs:1588-1602) and argmin over all candidates."""
import os
import socket

import numpy as np
import pytest

import oracle as O
from lewm_b200 import fleet as F

torch = pytest.importorskip("torch")


def test_split_range_covers_exactly():
    for n in (1, 7, 4096, 4099):
        for parts in (1, 2, 3, 8):
            if parts > n:
                continue
            ranges = [F.split_range(n, parts, i) for i in range(parts)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [r[1] - r[0] for r in ranges]
            assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("vehicles, samples, world, mode, expect", [
    (256, 4096, 8, "auto", (8, 1)),
    (256, 4096, 1, "auto", (1, 1)),
    (1, 4096, 8, "auto", (1, 8)),
    (2, 4096, 8, "auto", (2, 4)),
    (3, 512, 4, "auto", (2, 2)),
    (256, 4096, 4, "candidates", (1, 4)),
    (256, 4096, 4, "vehicles", (4, 1)),
])
def test_grid(vehicles, samples, world, mode, expect):
    assert F.grid(vehicles, samples, world, mode) == expect


def test_partition_groups_and_ranges():
    parts = F.partition(3, 10, 4, "auto")  # Gv = 2, Gs = 2
    assert [p.vehicles for p in parts] == [(0, 2), (0, 2), (2, 3), (2, 3)]
    assert [p.samples for p in parts] == [(0, 5), (5, 10), (0, 5), (5, 10)]
    assert [p.group_ranks for p in parts] == [(0, 1), (0, 1), (2, 3), (2, 3)]


def test_grid_rejects_impossible_splits():
    with pytest.raises(ValueError):
        F.grid(2, 16, 4, "vehicles")
    with pytest.raises(ValueError):
        F.grid(1, 2, 4, "candidates")
    with pytest.raises(ValueError):
        F.grid(4, 16, 2, "diagonal")


# ---- numpy restatement of the per-shard tuple (lwm_mppi.cuh) -------------

def _keys(scores, first_index):
    v = np.where(np.isnan(scores), np.float32(np.inf), scores).astype(np.float32)
    v = np.where(v == 0, np.float32(0), v).astype(np.float32)
    bits = v.view(np.uint32)
    hi = np.where(bits & np.uint32(0x80000000), ~bits, bits | np.uint32(0x80000000)).astype(np.uint64)
    idx = np.arange(scores.shape[-1], dtype=np.uint64) + np.uint64(first_index)
    return (hi << np.uint64(32)) | idx


def _key_score(key):
    hi = (key >> np.uint64(32)).astype(np.uint32)
    raw = np.where(hi & np.uint32(0x80000000), hi & np.uint32(0x7FFFFFFF), ~hi).astype(np.uint32)
    return raw.view(np.float32)


def shard_tuples(scores, cand, s0, temperature):
    """scores [B,s], cand [B,s,T,A] of samples [s0, s0+s) -> [B, 4 + T*A] f32."""
    B, s, T, A = cand.shape
    mul = np.float32(-1.0 / temperature)
    keys = _keys(scores, s0)
    best = keys.min(axis=1)
    m = _key_score(best)
    w = np.exp((scores - m[:, None]) * mul).astype(np.float32)
    out = np.zeros((B, 4 + T * A), np.float32)
    out[:, 0] = m
    out[:, 1] = w.sum(axis=1)
    out[:, 2:4] = best.view(np.float32).reshape(B, 2)
    out[:, 4:] = np.einsum("bs,bse->be", w, cand.reshape(B, s, T * A))
    return out


def combine(tuples, temperature):
    keys = np.ascontiguousarray(tuples[:, :, 2:4]).view(np.uint64)[..., 0]
    best = keys.min(axis=0)
    M = _key_score(best)
    f = np.exp((tuples[:, :, 0] - M[None]) * np.float32(-1.0 / temperature))
    W = (tuples[:, :, 1] * f).sum(axis=0)
    V = (tuples[:, :, 4:] * f[:, :, None]).sum(axis=0)
    return V / W[:, None], (best & np.uint64(0xFFFFFFFF)).astype(np.int64)


def _problem(vehicles, samples, seed=11):
    rng = np.random.default_rng(seed)
    T, A = 6, 4
    cand = rng.uniform(-1, 1, (vehicles, samples, T, A)).astype(np.float32)
    scores = (rng.standard_normal((vehicles, samples)) ** 2 * 5).astype(np.float32)
    scores[0, 3] = np.float32(np.nan)      # ranks as +inf, as in the reference
    scores[-1, samples // 2] = scores[-1].min()  # a tie across shards: the lower index wins
    return cand, scores


def _worker(rank, world, port, vehicles, samples, mode, temperature):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        parts = F.partition(vehicles, samples, world, mode)
        group = F.new_groups(parts)
        me = parts[rank]
        cand, scores = _problem(vehicles, samples)
        (v0, v1), (s0, s1) = me.vehicles, me.samples
        local = torch.from_numpy(shard_tuples(scores[v0:v1, s0:s1], cand[v0:v1, s0:s1], s0, temperature))
        if me.candidate_shards > 1:
            gathered = F.exchange_tuples(local, group, me.candidate_shards).numpy()
        else:
            gathered = local.numpy()[None]
        seq, best = combine(gathered, temperature)
        want = O.mppi_weighted(cand[v0:v1], scores[v0:v1], temperature).reshape(v1 - v0, -1)
        np.testing.assert_allclose(seq, want, rtol=1e-5, atol=1e-6)
        safe = np.where(np.isnan(scores[v0:v1]), np.inf, scores[v0:v1])
        assert (best == safe.argmin(axis=1)).all()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world, vehicles, samples, mode", [
    (2, 3, 64, "candidates"),
    (4, 2, 50, "auto"),       # 2 vehicle groups x 2 candidate shards
])
def test_sharded_mppi_equals_unsharded_over_gloo(world, vehicles, samples, mode):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(world, _free_port(), vehicles, samples, mode, 0.7), nprocs=world, join=True)


def _leaving_worker(rank, world, port, result_path):
    """Rank 1 leaves the job between two plan steps (its process exits); the
    other rank's next exchange fails within the process group's timeout and
    reports NCCL_ERROR instead of waiting for good."""
    import datetime
    import time as _time
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    from lewm_b200 import LwmError
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    parts = F.partition(2, 64, world, "candidates")
    group = F.new_groups(parts)
    me = parts[rank]
    cand, scores = _problem(2, 64)
    (s0, s1) = me.samples
    local = torch.from_numpy(shard_tuples(scores[:, s0:s1], cand[:, s0:s1], s0, 0.7))
    F.exchange_tuples_checked(local, group, world)  # plan step 1: every rank takes part
    if rank == 1:
        os._exit(0)  # leaves between plan steps, with no collective in flight
    t0 = _time.monotonic()
    try:
        F.exchange_tuples_checked(local, group, world)  # plan step 2: the peer is gone
        outcome = "no error"
    except LwmError as e:
        outcome = f"{e.status} after {_time.monotonic() - t0:.1f}s"
    with open(result_path, "w") as f:
        f.write(outcome)
    os._exit(0)  # the group cannot be torn down collectively without the peer


def test_rank_leaving_between_plan_steps_fails_the_next_exchange(tmp_path):
    import torch.multiprocessing as mp
    out = tmp_path / "outcome.txt"
    mp.spawn(_leaving_worker, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    outcome = out.read_text()
    assert outcome.startswith("NCCL_ERROR"), outcome
    assert float(outcome.split()[-1][:-1]) < 30.0, outcome
