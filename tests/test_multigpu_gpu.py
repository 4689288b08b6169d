"""Data-parallel training step on two GPUs (one process per GPU, NCCL).

The per-layer gradient buckets are summed over NCCL on a side stream,
overlapped with the backward, and SGD applies lr / 2 to the sum.
  - Same batch on both ranks: the sum is exactly twice each rank's gradient
    and (lr / 2) * (2 g) == lr * g in fp32, so the parameters must equal a
    single-GPU step bit for bit.
  - A different batch per rank: the summed gradient must equal g0 + g1
    recomputed locally (an allreduce that only doubled the rank's own
    gradient fails this), and the step must match a single-GPU step on the
    concatenated batch of 2B sequences within fp32 reassociation.
  - A rank that leaves between steps: it takes no part in the next step
    (none of its kernels or collectives in flight, its process alive); the
    other rank's next step ends with BWPP_CUDA_ERR_TIMEOUT within the
    communicator's 3 s bound (its watchdog aborts the NCCL communicator), and
    its context stays usable.  NVLS is off (NCCL_NVLS_ENABLE=0).
Needs two GPUs (skipped otherwise)."""
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


def _rank_distinct(rank, world, port, q):
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
        batches = []
        for r in range(world):  # every rank can regenerate every rank's batch
            g = torch.Generator(device="cuda").manual_seed(100 + r)
            batches.append((torch.randn(B * S, D, device="cuda", generator=g),
                            torch.randn(B * S, D, device="cuda", generator=g)))
        x, tgt = batches[rank]
        dp = bwpp.TinyModel(ctx, L, D, H, F, B, S, 1e-5, seed=3)
        solo = bwpp.TinyModel(ctx, L, D, H, F, B, S, 1e-5, seed=3)
        cat = bwpp.TinyModel(ctx, L, D, H, F, world * B, S, 1e-5, seed=3)
        n = dp.count
        # (1) the summed gradient against a local sum of both ranks' gradients
        dp.step(x, tgt, lr=0.0, comm=comm)
        g_dp = torch.empty(n, device="cuda")
        dp.get(None, g_dp)
        g_sum = torch.zeros(n, device="cuda")
        for r in range(world):
            solo.step(*batches[r], lr=0.0)
            gr = torch.empty(n, device="cuda")
            solo.get(None, gr)
            g_sum += gr
        ar_err = float(torch.linalg.norm((g_dp - g_sum).double()) / torch.linalg.norm(g_sum.double()))
        own = torch.empty(n, device="cuda")
        solo.step(x, tgt, lr=0.0)
        solo.get(None, own)
        own_err = float(torch.linalg.norm((g_dp - world * own).double()) / torch.linalg.norm(g_sum.double()))
        # (2) one step with lr against a single-GPU step on the concatenated batch
        p0 = torch.empty(n, device="cuda")
        dp.get(p0, None)
        dp.step(x, tgt, lr=0.1, comm=comm)
        p_dp = torch.empty(n, device="cuda")
        dp.get(p_dp, None)
        cat.step(torch.cat([b[0] for b in batches]), torch.cat([b[1] for b in batches]), lr=0.1)
        p_cat = torch.empty(n, device="cuda")
        cat.get(p_cat, None)
        # weights of magnitude ~0.1: one fp32 rounding is ~7e-9, far below
        # what a wrong gradient sum would move them
        step_err = float((p_dp - p_cat).abs().max())
        moved = float((p_dp - p0).abs().max())
        ctx.sync()
        lib.bwpp_cuda_comm_destroy(comm)
        for m in (dp, solo, cat):
            m.close()
        ctx.close()
        dist.destroy_process_group()
        q.put((rank, (ar_err, own_err, step_err, moved)))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)[:300]))


def _rank_leaves(rank, world, port, q, handled):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    try:
        import time

        import torch.distributed as dist
        import bwpp
        from bwpp.dist import comm_from_process_group
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        lib = bwpp.load()
        ctx = bwpp.Ctx(rank)
        L, D, H, F, B, S = 2, 256, 2, 512, 2, 256
        comm = comm_from_process_group(lib, rank, world, rank, dist, timeout_ms=3000)
        g = torch.Generator(device="cuda").manual_seed(40 + rank)
        x = torch.randn(B * S, D, device="cuda", generator=g)
        tgt = torch.randn(B * S, D, device="cuda", generator=g)
        model = bwpp.TinyModel(ctx, L, D, H, F, B, S, 1e-5, seed=3)
        model.step(x, tgt, lr=0.1, comm=comm)  # step 1: both ranks
        ctx.sync()
        assert lib.bwpp_cuda_comm_wait(comm) == bwpp.OK
        dist.barrier()
        if rank == 1:
            # leaves: no step 2; stays alive (its memory still mapped) until
            # the other rank has dealt with it
            handled.wait(timeout=120)
            lib.bwpp_cuda_comm_destroy(comm)
            model.close()
            ctx.close()
            q.put((rank, "left"))
            return
        t0 = time.monotonic()
        status = bwpp.OK
        try:
            model.step(x, tgt, lr=0.1, comm=comm)  # step 2: the peer never joins
            ctx.sync()
            status = lib.bwpp_cuda_comm_wait(comm)
        except bwpp.BwppError as e:
            status = e.status
        elapsed = time.monotonic() - t0
        aborted = lib.bwpp_cuda_comm_aborted(comm)
        ctx.sync()  # the NCCL kernels ended with the abort; the stream drains
        # the context still runs kernels
        a = torch.randn(256, 256, device="cuda").to(torch.bfloat16)
        c = torch.empty(256, 256, device="cuda")
        ctx.matmul_bf16(a, a, c, 256, 256, 256, 256, 256, 256, None, 0, 0)
        ctx.sync()
        ok = bool(torch.allclose(c, a.float() @ a.float(), rtol=1e-2, atol=1e-2))
        handled.set()
        lib.bwpp_cuda_comm_destroy(comm)
        model.close()
        ctx.close()
        q.put((rank, (status, elapsed, aborted, ok)))
    except Exception as e:  # reported to the parent
        handled.set()
        q.put((rank, repr(e)[:300]))


def test_two_gpu_rank_leaving_between_steps_times_out_the_next_step():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    handled = ctx.Event()
    port = _free_port()
    procs = [ctx.Process(target=_rank_leaves, args=(r, 2, port, q, handled)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, out = q.get(timeout=300)
        res[r] = out
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1] == "left", res
    import bwpp
    status, elapsed, aborted, ok = res[0]
    assert status == bwpp.ERR_TIMEOUT, res
    assert 2.5 <= elapsed <= 30.0, res  # the 3 s bound, not a hang
    assert aborted == 1 and ok, res


def _rank_matmul_dist(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        import numpy as np
        import torch.distributed as dist
        import bwpp
        import oracle as O
        from bwpp.dist import comm_from_process_group, split_rows
        torch.cuda.set_device(rank)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        lib = bwpp.load()
        comm = comm_from_process_group(lib, rank, world, rank, dist)
        M, K, N = 700, 1000, 1032  # K split 500 / 500, M unevenly
        rng = np.random.default_rng(5)
        a = (0.1 * rng.standard_normal((M, K))).astype(np.float32)
        b = (0.1 * rng.standard_normal((K, N))).astype(np.float32)
        bias = rng.uniform(-0.1, 0.1, N).astype(np.float32)
        r0, r1 = split_rows(M, rank, world)
        ha = torch.from_numpy(np.ascontiguousarray(a[r0:r1])).pin_memory()
        hb, hbias = torch.from_numpy(b).pin_memory(), torch.from_numpy(bias).pin_memory()
        errs = []
        for _ in range(2):
            hc = torch.full((r1 - r0, N), float("nan")).pin_memory()
            bwpp.matmul_f32_dist(comm, ha, hb, hc, r1 - r0, N, K, K, N, N, hbias, 1, 1)
            ref = O.matmul(O.bf16_to_f32(O.f32_to_bf16(a[r0:r1])), O.bf16_to_f32(O.f32_to_bf16(b)),
                           bias, 1, 1)
            d = hc.numpy() - ref
            errs.append(float(np.linalg.norm(d) / np.linalg.norm(ref)))
        lib.bwpp_cuda_comm_destroy(comm)
        dist.destroy_process_group()
        q.put((rank, errs))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)[:300]))


def test_two_gpu_f32_matmul_mirror_with_all_gathered_w():
    """bwpp_cuda_matmul_f32_dist: each rank uploads half of W's K rows, the
    bf16 W is all-gathered over NCCL, each rank's C rows match the oracle on
    the bf16-rounded operands (1e-2 north-star bound, 2e-4 bug detector)."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = _run_two(_rank_matmul_dist)
    for r in range(2):
        assert isinstance(res[r], list), res
        assert max(res[r]) <= 2e-4, res


def _run_two(target):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        r, out = q.get(timeout=300)
        res[r] = out
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return res


def test_two_gpu_data_parallel_step_distinct_batches():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    res = _run_two(_rank_distinct)
    for r in range(2):
        assert isinstance(res[r], tuple), res
        ar_err, own_err, step_err, moved = res[r]
        assert ar_err <= 1e-6, res          # NCCL sum == g0 + g1 (two operands: exact)
        assert own_err >= 1e-2, res         # and not world x the local gradient
        assert step_err <= 1e-6, res        # same weights as the concatenated-batch step
        assert moved > 1e-5, res            # which did move them


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
