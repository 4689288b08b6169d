"""Multi-rank host logic with world_size-2 gloo process groups on CPU.

Covers what the GPU runs do between ranks: the row / head sharding of every
sharded config (no collective on the data path), the byte broadcast that
bootstraps the NCCL communicator of the training step, the max-over-ranks
timing, and failure handling: a rank that leaves without joining a
collective makes the other rank's next collective end with an error after a
short process-group timeout instead of hanging.  No GPU is involved.
"""
import datetime
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from bwpp.dist import broadcast_bytes, max_over_ranks, split_rows


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def run_ranks(fn, world, *args):
    port = free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    deadline = time.time() + 120
    while len(results) < world and time.time() < deadline:
        try:
            r, val = q.get(timeout=5)
            results[r] = val
        except Exception:
            if all(not p.is_alive() for p in procs) and q.empty():
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return results


def _entry(fn, rank, world, port, q, *args):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        q.put((rank, fn(rank, world, *args)))
    except Exception as e:  # reported to the parent, not raised in the child
        q.put((rank, ("error", type(e).__name__, str(e)[:200])))


def _shards(rank, world):
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=30))
    out = {}
    for name, total in (("gemm_rows", 8192), ("attention_heads", 8 * 32), ("norm_rows", 65536),
                        ("odd", 7)):
        mine = torch.tensor(split_rows(total, rank, world))
        gathered = [torch.zeros(2, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(gathered, mine)
        out[name] = [tuple(g.tolist()) for g in gathered]
    payload = broadcast_bytes(bytes(range(128)) if rank == 0 else None, dist)
    out["uid_ok"] = payload == bytes(range(128))
    out["max"] = max_over_ranks(1.5 + rank, dist)
    dist.destroy_process_group()
    return out


def test_sharding_broadcast_and_max_over_ranks_gloo():
    res = run_ranks(_shards, 2)
    assert set(res) == {0, 1}, res
    for r in (0, 1):
        assert isinstance(res[r], dict), res[r]
        assert res[r]["uid_ok"]
        assert res[r]["max"] == 2.5
    for name, total in (("gemm_rows", 8192), ("attention_heads", 256), ("norm_rows", 65536), ("odd", 7)):
        shards = res[0][name]
        assert shards == res[1][name]
        # contiguous, disjoint, covering [0, total)
        assert shards[0][0] == 0 and shards[-1][1] == total
        assert all(a[1] == b[0] for a, b in zip(shards, shards[1:]))
        sizes = [b - a for a, b in shards]
        assert max(sizes) - min(sizes) <= 1


def test_split_rows_single_process_edges():
    assert split_rows(10, 0, 1) == (0, 10)
    assert [split_rows(3, r, 4) for r in range(4)] == [(0, 1), (1, 2), (2, 3), (3, 3)]
    with pytest.raises(ValueError):
        split_rows(10, 2, 2)


def _dropout(rank, world):
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    t = torch.ones(4)
    dist.all_reduce(t)  # one good step on both ranks
    if rank == 1:
        return "left"  # leaves between steps: never joins the next collective
    t0 = time.time()
    try:
        dist.all_reduce(t)
        return ("no error", time.time() - t0)
    except Exception as e:
        return ("error", type(e).__name__, round(time.time() - t0, 1))


def test_rank_that_leaves_makes_the_next_collective_fail_fast():
    res = run_ranks(_dropout, 2)
    assert res.get(1) == "left", res
    r0 = res.get(0)
    assert isinstance(r0, tuple) and r0[0] == "error", r0
    assert r0[-1] < 60, r0
