"""Multi-rank host logic on CPU (gloo, world size 2 and 4): head / sequence sharding,
LPT balance and reassembly of the gathered outputs, and a rank that fails before
the collective (the others see an error, nothing hangs)."""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "kitty-kv_b200"))

from kitty.distributed import (gather_head_outputs, gather_sequence_outputs, kv_head_range, lpt_assign,  # noqa: E402
                               q_head_range, sequence_costs)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fn, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        q.put((rank, "ok", fn(rank, world)))
    except Exception as e:  # report, then leave the group
        q.put((rank, "error", repr(e)))
    finally:
        dist.destroy_process_group()


def _run(world, fn):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fn, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, status, val = q.get(timeout=120)
        results[rank] = (status, val)
    for p in procs:
        p.join(timeout=60)
    return results


def full_output(B, Hq, D):
    g = torch.Generator().manual_seed(0)
    return torch.randn(B, Hq, D, generator=g)


def head_sharded(rank, world):
    B, Hq, H, D = 3, 16, 4, 8
    full = full_output(B, Hq, D)
    q0, q1 = q_head_range(Hq, H, world, rank)
    local = full[:, q0:q1].permute(1, 0, 2).contiguous()        # head-major local output
    got = gather_head_outputs(local)
    return bool(torch.equal(got, full))


def seq_sharded(rank, world):
    B, Hq, D = 7, 4, 8
    full = full_output(B, Hq, D)
    costs = [float(x) for x in (5, 1, 9, 3, 3, 7, 2)]
    assignment = lpt_assign(costs, world)
    local = full[assignment[rank]] if assignment[rank] else torch.zeros(0, Hq, D)
    got = gather_sequence_outputs(local, assignment)
    return bool(torch.equal(got, full))


@pytest.mark.parametrize("world", [2, 4])
def test_head_sharded_gather(world):
    res = _run(world, head_sharded)
    assert all(s == "ok" and v for s, v in res.values()), res


@pytest.mark.parametrize("world", [2, 4])
def test_sequence_sharded_gather(world):
    res = _run(world, seq_sharded)
    assert all(s == "ok" and v for s, v in res.values()), res


def failing_rank(rank, world):
    if rank == 1:
        raise RuntimeError("rank 1 failed before the collective")
    # the surviving rank's collective must end with an error, not hang
    t = torch.zeros(4)
    dist.all_reduce(t)
    return True


def test_failed_rank_does_not_hang():
    res = _run(2, failing_rank)
    assert res[1][0] == "error" and "rank 1 failed" in res[1][1]
    assert res[0][0] == "error"        # peer left: gloo reports a connection error


def test_partition_helpers():
    assert kv_head_range(8, 4, 3) == (6, 8)
    assert q_head_range(64, 8, 8, 2) == (16, 24)
    with pytest.raises(ValueError):
        kv_head_range(8, 3, 0)
    bins = lpt_assign([10, 9, 8, 7, 1, 1], 2)
    loads = [sum([10, 9, 8, 7, 1, 1][i] for i in b) for b in bins]
    assert sorted(sum(bins, [])) == list(range(6)) and max(loads) - min(loads) <= 2
    c = sequence_costs([2, 0], [32, 4], [5, 0], 8, 9728, 128)
    assert c == [8 * (2 * 9728 + 37 * 512), 8 * (4 * 512)]
