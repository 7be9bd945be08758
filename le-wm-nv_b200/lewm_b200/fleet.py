"""Fleet planning across the GPUs of one node (one process per GPU).

A fleet is B independent vehicles, each planning S candidates x T steps with
its own context and physical parameters.  The ranks form a Gv x Gs grid:

* vehicle groups (Gv): vehicles are split into Gv contiguous ranges; the
  groups never communicate (planning is independent per vehicle);
* candidate shards (Gs): inside a vehicle group the S candidates are split
  into Gs contiguous ranges.  Each shard scores its range and reduces it to
  one MPPI tuple per vehicle (min score, sum of weights, best key, weighted
  action sums); one all-gather of those tuples over the group (NCCL over
  NVLink, B x (4 + T*A) floats per GPU) and a combine kernel finish the plan
  identically on every shard, warm start included.

Every shard draws the same Philox noise as a single-GPU planner over all S
candidates, so the sharded plan equals the unsharded one up to the order of
the floating-point sums.  The rotor-forces integrator takes each vehicle's
mass (src/models/skyjepa/kinematics.rs:411-413); the reference would need one
scorer per vehicle.
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

MODES = ("auto", "vehicles", "candidates")


def split_range(n: int, parts: int, index: int) -> Tuple[int, int]:
    """Contiguous range `index` of `parts` near-equal ranges of [0, n)."""
    if parts <= 0 or not 0 <= index < parts:
        raise ValueError(f"range {index} of {parts} parts")
    base, extra = divmod(n, parts)
    start = index * base + min(index, extra)
    return start, start + base + (1 if index < extra else 0)


@dataclass(frozen=True)
class FleetPart:
    rank: int
    vehicle_groups: int       # Gv
    candidate_shards: int     # Gs
    vehicle_group: int
    candidate_shard: int
    vehicles: Tuple[int, int]  # [v0, v1)
    samples: Tuple[int, int]   # [s0, s1)
    group_ranks: Tuple[int, ...]  # ranks sharing this vehicle range (the all-gather group)


def grid(vehicles: int, samples: int, world: int, mode: str = "auto") -> Tuple[int, int]:
    """(Gv, Gs) for `world` ranks."""
    if mode not in MODES:
        raise ValueError(f"unknown shard mode {mode!r}; expected one of {MODES}")
    if world < 1 or vehicles < 1 or samples < 1:
        raise ValueError("world, vehicles and samples must be positive")
    if mode == "vehicles":
        if world > vehicles:
            raise ValueError(f"{world} ranks cannot split {vehicles} vehicles")
        return world, 1
    if mode == "candidates":
        if world > samples:
            raise ValueError(f"{world} ranks cannot split {samples} candidates")
        return 1, world
    # auto: as many vehicle groups as possible (no exchange), the rest by candidates
    gv = max(d for d in range(1, world + 1) if world % d == 0 and d <= vehicles)
    gs = world // gv
    if gs > samples:
        raise ValueError(f"{world} ranks cannot split {vehicles} vehicles x {samples} candidates")
    return gv, gs


def partition(vehicles: int, samples: int, world: int, mode: str = "auto") -> List[FleetPart]:
    gv, gs = grid(vehicles, samples, world, mode)
    parts = []
    for rank in range(world):
        vg, cs = divmod(rank, gs)
        parts.append(FleetPart(rank, gv, gs, vg, cs, split_range(vehicles, gv, vg), split_range(samples, gs, cs),
                               tuple(range(vg * gs, vg * gs + gs))))
    return parts


def new_groups(parts: Sequence[FleetPart]):
    """One process group per vehicle group with more than one shard.  Every
    rank calls this with the same parts (torch.distributed.new_group is
    collective over the default group); returns this rank's group or None."""
    import torch.distributed as dist
    rank = dist.get_rank()
    mine = None
    seen = []
    for p in parts:
        if p.group_ranks in seen:
            continue
        seen.append(p.group_ranks)
        if len(p.group_ranks) > 1:
            g = dist.new_group(list(p.group_ranks))
            if rank in p.group_ranks:
                mine = g
    return mine


def exchange_tuples(local, group, shards: int, out=None):
    """All-gather this shard's [B, width] tuples into [shards, B, width] over
    `group` (the ranks sharing the vehicle range)."""
    import torch
    import torch.distributed as dist
    if out is None:
        out = torch.empty((shards,) + tuple(local.shape), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    else:  # gloo (host tensors): gather into views of the same buffer
        dist.all_gather(list(out.unbind(0)), local.contiguous(), group=group)
    return out


def exchange_tuples_checked(local, group, shards: int, out=None):
    """exchange_tuples whose failure — a rank of the vehicle group that left,
    or a collective that ran out the process group's timeout (the bounded
    wait of the exchange) — surfaces as LwmError with status NCCL_ERROR, so a
    caller can drop the group and re-plan on the ranks that remain."""
    from . import LwmError
    try:
        return exchange_tuples(local, group, shards, out=out)
    except Exception as e:  # gloo / NCCL raise RuntimeError subclasses (or DistBackendError)
        raise LwmError(4, f"candidate-shard tuple exchange over {shards} ranks failed "
                          f"({type(e).__name__}: {str(e).splitlines()[0] if str(e) else ''})") from e


class FleetPlanner:
    """One rank's share of a fleet: a learned (SkyJEPA) or nominal scorer over
    its vehicle range and an MPPI planner over its candidate range."""

    def __init__(self, ctx, part: FleetPart, scorer, mppi_config, group=None, time_exchange: bool = False):
        """`time_exchange`: record CUDA events around every tuple exchange on
        the context's stream (exchange_ms() reads them back)."""
        import torch
        from . import MppiPlanner
        self.ctx = ctx
        self.part = part
        self.scorer = scorer
        self.group = group
        self.time_exchange = time_exchange
        self._events = []
        s0, s1 = part.samples
        self.planner = MppiPlanner(ctx, dataclasses.replace(mppi_config, samples=s1 - s0))
        self.sharded = part.candidate_shards > 1
        if self.sharded:
            self.planner.set_shard(s0, mppi_config.samples)
        self._gathered = None
        self._torch = torch

    def plan_device(self):
        """Plan every vehicle of this rank's range; returns a PlanDeviceResult
        whose sequence/first_action are the fleet-wide (all-shard) result."""
        if not self.sharded:
            return self.planner.plan_device(self.scorer)
        from . import device_tensor
        torch = self._torch
        ptr, width = self.planner.plan_device_shard(self.scorer)
        B = self.scorer.batch
        local = device_tensor(ptr, (B, width))
        if self._gathered is None or self._gathered.shape != (self.part.candidate_shards, B, width):
            self._gathered = torch.empty((self.part.candidate_shards, B, width), dtype=torch.float32,
                                         device=local.device)
        stream = self.ctx.torch_stream()
        with torch.cuda.stream(stream):
            if self.time_exchange:
                ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                ev[0].record(stream)
            exchange_tuples_checked(local, self.group, self.part.candidate_shards, out=self._gathered)
            if self.time_exchange:
                ev[1].record(stream)
                self._events.append(ev)
        return self.planner.combine_device(self._gathered.data_ptr(), self.part.candidate_shards)

    def exchange_ms(self, clear: bool = True):
        """Device time of every timed tuple exchange since the last call (ms)."""
        out = []
        for s, e in self._events:
            e.synchronize()
            out.append(s.elapsed_time(e))
        if clear:
            self._events = []
        return out

    def close(self) -> None:
        self.planner.close()



def nccl_elite_exchange(ctx, group, shards: int):
    """The exchange of CEM / iCEM candidate shards (IcemPlanner.set_shard_exchange)
    as one NCCL all-gather over `group` on the context's stream."""
    import torch
    import torch.distributed as dist
    from . import device_tensor

    def exchange(local_ptr, count, gathered_ptr, _stream):
        src = device_tensor(local_ptr, (count,))
        dst = device_tensor(gathered_ptr, (shards * count,))
        with torch.cuda.stream(ctx.torch_stream()):
            dist.all_gather_into_tensor(dst, src, group=group)
    return exchange
