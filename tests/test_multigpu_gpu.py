"""Data-parallel training step on two GPUs (one process per GPU, NCCL).

Both ranks step the same tiny_model on the same batch; the per-layer
gradient buckets are summed over NCCL on a side stream, overlapped with the
backward, and SGD applies lr / 2 to the sum.  With identical data the sum is
exactly twice each rank's gradient and (lr / 2) * (2 g) == lr * g in fp32,
so the parameters must equal a single-GPU step bit for bit.  Needs two GPUs
(skipped otherwise)."""
import datetime
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        import torch.distributed as dist
        import bwpp
        from bwpp.dist import comm_from_process_group
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        lib = bwpp.load()
        ctx = bwpp.Ctx(rank)
        L, D, H, F, B, S = 2, 256, 2, 512, 2, 256
        comm = comm_from_process_group(lib, rank, world, rank, dist)
        g = torch.Generator(device="cuda").manual_seed(11)
        x = torch.randn(B * S, D, device="cuda", generator=g)
        tgt = torch.randn(B * S, D, device="cuda", generator=g)
        dp = bwpp.TinyModel(ctx, L, D, H, F, B, S, 1e-5, seed=3)
        solo = bwpp.TinyModel(ctx, L, D, H, F, B, S, 1e-5, seed=3)
        for _ in range(2):
            dp.step(x, tgt, lr=0.1, comm=comm)
            solo.step(x, tgt, lr=0.1)
        p_dp = torch.empty(dp.count, device="cuda")
        p_solo = torch.empty(solo.count, device="cuda")
        dp.get(p_dp, None)
        solo.get(p_solo, None)
        ctx.sync()
        diff = float((p_dp - p_solo).abs().max())
        lib.bwpp_cuda_comm_destroy(comm)
        dp.close()
        solo.close()
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, diff))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)[:300]))


def test_two_gpu_data_parallel_step_matches_single_gpu():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, diff = q.get(timeout=300)
        res[r] = diff
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[0] == 0.0 and res[1] == 0.0, res
