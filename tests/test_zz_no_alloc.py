"""bwpp_cuda_rmsnorm_bwd_f32_noalloc: the RMSNorm backward for callers that
cannot allocate device memory (a host framework that owns the whole device
memory budget, or a latency-critical loop that must not cudaMalloc / cudaFree).
Its scratch is a fixed array inside the library.  Checked through the C ABI
against the allocating entry point, bwpp_cuda_rmsnorm_bwd_f32, on two calls in
a row.  Collected last on purpose; it also passes alone in a fresh process."""
import numpy as np
import pytest
import torch

import bwpp
from conftest import rel_fro

pytestmark = pytest.mark.gpu
TOL = 1e-5  # the norm tolerance of the other GPU tests


def _inputs(seed, rows, cols):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, cols, device="cuda", generator=g)
    dy = torch.randn(rows, cols, device="cuda", generator=g)
    gamma = 1 + 0.1 * torch.randn(cols, device="cuda", generator=g)
    return x, dy, gamma


@pytest.mark.parametrize("rows,cols", [(4096, 4096), (300, 1000), (7, 20000)])
def test_noalloc_matches_allocating_entry_point(rows, cols):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    lib = bwpp.load()
    ctx = bwpp.Ctx(0)
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((11, 12)):  # two calls in a row, different inputs
        x, dy, gamma = _inputs(seed + rows, rows, cols)
        ref_dx, ref_dg, ref_db = torch.empty_like(x), torch.empty(cols, device="cuda"), torch.empty(cols, device="cuda")
        ctx.rmsnorm_bwd(x, gamma, dy, ref_dx, ref_dg, ref_db, rows, cols, cols, 1e-5)
        ctx.sync()
        dx = torch.full_like(x, float("nan"))
        dg = torch.full((cols,), float("nan"), device="cuda")
        db = torch.full((cols,), float("nan"), device="cuda")
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        rc = lib.bwpp_cuda_rmsnorm_bwd_f32_noalloc(x.data_ptr(), gamma.data_ptr(), dy.data_ptr(),
                                                   dx.data_ptr(), dg.data_ptr(), db.data_ptr(),
                                                   rows, cols, cols, 1e-5, stream)
        assert rc == bwpp.OK, (call, rc)
        torch.cuda.synchronize()
        assert torch.cuda.mem_get_info()[0] == free0  # nothing allocated
        assert rel_fro(dx.cpu().numpy(), ref_dx.cpu().numpy()) <= TOL, call
        assert rel_fro(dg.cpu().numpy(), ref_dg.cpu().numpy()) <= TOL, call
        assert rel_fro(db.cpu().numpy(), ref_db.cpu().numpy()) <= TOL, call
    ctx.close()


def test_noalloc_rejects_rows_wider_than_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    lib = bwpp.load()
    cols = 524288 + 4  # 2 * cols floats exceed the 1,048,576-float scratch
    x = torch.zeros(1, cols, device="cuda")
    rc = lib.bwpp_cuda_rmsnorm_bwd_f32_noalloc(x.data_ptr(), None, x.data_ptr(), x.data_ptr(),
                                               x.data_ptr(), None, 1, cols, cols, 1e-5, None)
    assert rc == bwpp.ERR_ARG
    # without dgamma / dbeta no scratch is needed and the same width runs
    dx = torch.empty_like(x)
    rc = lib.bwpp_cuda_rmsnorm_bwd_f32_noalloc(x.data_ptr(), None, x.data_ptr(), dx.data_ptr(),
                                               None, None, 1, cols, cols, 1e-5, None)
    assert rc == bwpp.OK
    torch.cuda.synchronize()
