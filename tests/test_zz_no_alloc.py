"""bwpp_cuda_rmsnorm_bwd_f32_noalloc: the RMSNorm backward for callers that
cannot allocate device memory (a host framework that owns the whole device
memory budget, or a latency-critical loop that must not cudaMalloc / cudaFree).
Its scratch is a fixed array inside the library.  Checked through the C ABI
against the allocating entry point, bwpp_cuda_rmsnorm_bwd_f32, on two calls in
a row, and against the CPU oracle (oracle/, the restatement of the backward
rule of compiler/graph_ir.c:1735-1789).  Collected last on purpose; it also
passes alone in a fresh process."""
import numpy as np
import pytest
import torch

import bwpp
import oracle as O
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
        # and against the CPU oracle on the same inputs
        o_dx, o_dg, o_db = O.norm_bwd(x.cpu().numpy(), gamma.cpu().numpy(), dy.cpu().numpy(), 1e-5,
                                      False)
        assert rel_fro(dx.cpu().numpy(), o_dx) <= TOL, call
        assert rel_fro(dg.cpu().numpy(), o_dg) <= TOL, call
        assert rel_fro(db.cpu().numpy(), o_db) <= TOL, call
    ctx.close()


@pytest.mark.parametrize("rows,want", [(0, "both"), (513, "dgamma"), (513, "dbeta"), (0, "dbeta")])
def test_noalloc_partial_outputs_and_empty_rows(rows, want):
    """dgamma only, dbeta only, and rows = 0 (sums over no rows are 0, dx untouched)."""
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    lib = bwpp.load()
    ctx = bwpp.Ctx(0)
    cols = 1000
    stream = torch.cuda.current_stream().cuda_stream
    x, dy, gamma = _inputs(77, max(rows, 1), cols)
    x, dy = x[:rows].contiguous(), dy[:rows].contiguous()
    ref_dx = torch.empty_like(x)
    ref_dg, ref_db = torch.zeros(cols, device="cuda"), torch.zeros(cols, device="cuda")
    if rows:  # sums over no rows are 0
        ctx.rmsnorm_bwd(x, gamma, dy, ref_dx, ref_dg, ref_db, rows, cols, cols, 1e-5)
        ctx.sync()
    for _ in range(2):
        dx = torch.full_like(x, float("nan"))
        dg = torch.full((cols,), float("nan"), device="cuda")
        db = torch.full((cols,), float("nan"), device="cuda")
        pg = dg.data_ptr() if want in ("both", "dgamma") else None
        pb = db.data_ptr() if want in ("both", "dbeta") else None
        # with rows = 0 the row buffers are empty: a valid dummy stands in for them
        dummy = torch.zeros(4, device="cuda")
        px, pdy, pdx = ((t.data_ptr() if rows else dummy.data_ptr()) for t in (x, dy, dx))
        rc = lib.bwpp_cuda_rmsnorm_bwd_f32_noalloc(px, gamma.data_ptr(), pdy, pdx, pg, pb,
                                                   rows, cols, cols, 1e-5, stream)
        assert rc == bwpp.OK, rc
        torch.cuda.synchronize()
        if rows:
            assert rel_fro(dx.cpu().numpy(), ref_dx.cpu().numpy()) <= TOL
        if pg:
            assert rel_fro(dg.cpu().numpy(), ref_dg.cpu().numpy()) <= TOL
        else:
            assert bool(torch.isnan(dg).all())  # not requested, not written
        if pb:
            assert rel_fro(db.cpu().numpy(), ref_db.cpu().numpy()) <= TOL
        else:
            assert bool(torch.isnan(db).all())
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
