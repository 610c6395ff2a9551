"""Token-row sharding across the GPUs of one node (one process per GPU).

The ops of this path are independent per token row, so ranks exchange no data:
each rank processes a contiguous block of the token rows (or, for weak scaling,
its own full-size batch), and torch.distributed carries only control -- a
barrier, the max of the per-rank device times, and failure propagation so that
one rank's exception fails every rank at the same step instead of leaving the
others waiting.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    begin: int
    end: int

    @property
    def size(self) -> int:
        return self.end - self.begin


def shard_range(total: int, rank: int, world: int, align: int = 1) -> Shard:
    """Contiguous block of `total` units for `rank`: ceil(total/world) units per
    rank (rounded up to `align`), the last ranks possibly shorter or empty."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if total < 0 or align <= 0:
        raise ValueError("total must be >= 0 and align > 0")
    per = -(-total // world)
    per = -(-per // align) * align
    begin = min(total, rank * per)
    end = min(total, begin + per)
    return Shard(rank, world, begin, end)


class ShardFailure(RuntimeError):
    """Raised on every rank when any rank failed its step."""


def max_over_ranks(value: float, device=None) -> float:
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def run_step(fn, *args, device=None, **kwargs):
    """Runs fn on this rank, then agrees with every other rank on whether all
    succeeded. A failure anywhere raises ShardFailure on every rank after the
    local work has finished (no rank is left inside a collective)."""
    import torch
    import torch.distributed as dist
    err = None
    result = None
    try:
        result = fn(*args, **kwargs)
        if device is not None and torch.cuda.is_available():
            torch.cuda.synchronize(device)
    except Exception as e:  # reported to all ranks below
        err = e
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        flag = torch.tensor([1.0 if err is not None else 0.0], device=device)
        dist.all_reduce(flag, op=dist.ReduceOp.MAX)
        failed = flag.item() > 0
    else:
        failed = err is not None
    if failed:
        raise ShardFailure(f"a rank failed its step: {err!r}" if err else
                           "another rank failed its step") from err
    return result


def barrier(device=None) -> None:
    """Process-group barrier (no-op for a single process)."""
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        if device is not None and getattr(device, "type", None) == "cuda":
            dist.barrier(device_ids=[device.index])
        else:
            dist.barrier()


def timed_region(step, steps: int, *, start, stop, device=None):
    """The timed loop of a multi-rank benchmark: a barrier, then
    start(); step(0) .. step(steps-1); stop() on every rank, inside one
    run_step -- so the loop itself carries no collective, and a rank whose step
    raises makes every rank raise ShardFailure right after the loop instead of
    leaving the others blocked in the next collective. start/stop record the
    clock (CUDA events on the launching stream, or the host clock); run_step
    synchronises `device` before the ranks compare notes. Returns stop()'s
    result."""
    out = []

    def loop():
        start()
        for i in range(steps):
            step(i)
        out.append(stop())

    barrier(device)
    if device is not None:
        import torch
        torch.cuda.synchronize(device)
    run_step(loop, device=device)
    barrier(device)
    return out[0]
