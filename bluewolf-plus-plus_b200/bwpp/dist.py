"""Host-side logic of the multi-GPU paths (one process per GPU).

Work that shards naturally (GEMM rows, attention batch x head, norm and
reduce_max rows) is split with `split_rows` and needs no collective.  The
only data-path collective is the tiny_model gradient allreduce, whose NCCL
communicator is bootstrapped from an existing torch.distributed process group
by `comm_from_process_group` (rank 0 creates the NCCL id, the group
broadcasts it).  `max_over_ranks` turns per-rank device times into the
whole-job time.  Everything here is plain Python over torch.distributed, so
it is tested with gloo ranks on CPU.
"""
from __future__ import annotations

import ctypes as C


def split_rows(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous [start, end) share of `total` units for `rank` of `world`;
    the first total % world ranks get one extra unit."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    base, rem = divmod(total, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def broadcast_bytes(payload: bytes | None, dist, src: int = 0) -> bytes:
    """Broadcasts a bytes payload from `src` over the default process group."""
    obj = [payload]
    dist.broadcast_object_list(obj, src=src)
    return obj[0]


def comm_from_process_group(lib, rank: int, world: int, device: int, dist, timeout_ms: int = 120000):
    """Creates a BwppCudaComm for (rank, world): rank 0 makes the 128-byte
    NCCL id, the process group broadcasts it, every rank joins (bounded by
    timeout_ms, which also bounds every later wait on the communicator)."""
    uid = (C.c_ubyte * 128)()
    payload = None
    if rank == 0:
        rc = lib.bwpp_cuda_comm_unique_id(uid)
        if rc != 0:
            raise RuntimeError(f"bwpp_cuda_comm_unique_id failed ({rc})")
        payload = bytes(uid)
    payload = broadcast_bytes(payload, dist)
    uid = (C.c_ubyte * 128).from_buffer_copy(payload)
    handle = C.c_void_p()
    rc = lib.bwpp_cuda_comm_create_timeout(C.byref(handle), uid, rank, world, device, int(timeout_ms))
    if rc != 0:
        raise RuntimeError(f"bwpp_cuda_comm_create_timeout failed ({rc})")
    return handle


def max_over_ranks(value: float, dist, device="cpu") -> float:
    """Max of a per-rank float over the default group (identity without one)."""
    import torch
    if not (dist.is_available() and dist.is_initialized()):
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
