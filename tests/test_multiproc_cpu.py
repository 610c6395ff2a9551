"""Multi-rank host logic on CPU: gloo, world size 2, 127.0.0.1 rendezvous.

Covers the token-row shard split, the max-over-ranks timing reduction and
failure propagation (a rank that raises makes every rank raise at the same
step), without any GPU."""

import os
import socket

import pytest
import torch.multiprocessing as mp

from tfx.shard import ShardFailure, shard_range


def test_shard_ranges_cover_every_row_once():
    for total in (0, 1, 7, 32768, 32769):
        for world in (1, 2, 4, 8):
            for align in (1, 4):
                seen = []
                for r in range(world):
                    s = shard_range(total, r, world, align)
                    assert 0 <= s.begin <= s.end <= total
                    seen.extend(range(s.begin, s.end))
                assert seen == list(range(total))
    assert shard_range(32768, 3, 8).size == 4096
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fail_rank, out):
    import datetime
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "tenferro-decision-rs_b200"))
    import torch
    import torch.distributed as dist
    from tfx.shard import ShardFailure, max_over_ranks, run_step, shard_range

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    try:
        shard = shard_range(64, rank, world)
        x = torch.arange(shard.begin, shard.end, dtype=torch.float64)
        total = torch.tensor([x.sum().item()])
        dist.all_reduce(total)
        t = max_over_ranks(float(rank + 1) * 1.5)

        def step(i):
            if rank == fail_rank and i == 1:
                raise RuntimeError("injected host failure")
            return i

        results = []
        failed_at = None
        for i in range(3):
            try:
                results.append(run_step(step, i))
            except ShardFailure:
                failed_at = i
                break
        # the bench's timed loop: one region of several steps, no collective
        # inside it; a failing step fails every rank right after the region
        from tfx.shard import timed_region
        import time
        seen = []

        def region_step(i):
            seen.append(i)
            if rank == fail_rank and i == 2:
                raise RuntimeError("injected host failure in the timed region")

        box = {}
        try:
            ms = timed_region(region_step, 4,
                              start=lambda: box.__setitem__("t", time.perf_counter()),
                              stop=lambda: (time.perf_counter() - box["t"]) * 1e3)
            region = ("ok", ms >= 0.0, len(seen))
        except ShardFailure:
            region = ("failed", True, len(seen))
        out.put((rank, float(total.item()), t, results, failed_at, region))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("fail_rank", [-1, 1])
def test_gloo_world2_max_and_failure_propagation(fail_rank):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, fail_rank, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = sorted(out.get(timeout=10) for _ in procs)
    for rank, total, t, results, failed_at, region in got:
        assert total == sum(range(64))
        assert t == 3.0  # max of 1.5, 3.0
        if fail_rank < 0:
            assert results == [0, 1, 2] and failed_at is None
            assert region == ("ok", True, 4)
        else:
            assert results == [0] and failed_at == 1  # every rank stops at the failing step
            # every rank raises after the region; the failing rank stopped at its step
            assert region[0] == "failed"
            assert region[2] == (3 if rank == fail_rank else 4)
