"""f16 variants (the half ABI of the MSL kernels) on the GPU vs the CPU oracle.

Inputs are IEEE half (numpy float16, nearest even); the oracle runs in fp32
on their exact upcast (the same restatements of runtime/cpu/bwpp_cpu_ref.c
the bf16 / fp32 tests use).  Tolerances:
  contractions (matmul, attention): relative Frobenius <= 1e-2 (north star),
    and a tighter 2e-3 bug detector (one half rounding of the output is
    <= 2^-11 relative per element)
  softmax / rmsnorm: <= 1e-3 (their only error is the half rounding of y)
"""
import numpy as np
import pytest
import torch

import bwpp
import oracle as O
from conftest import rel_fro

pytestmark = pytest.mark.gpu
TOL_MM, TIGHT_MM, TOL_ROW = 1e-2, 2e-3, 1e-3


def half(rng, *shape, scale=1.0):
    return (scale * rng.standard_normal(shape)).astype(np.float16)


def d(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def h(t):
    return t.cpu().numpy().astype(np.float32)


@pytest.mark.parametrize("M,N,K", [(1, 8, 8), (3, 40, 24), (128, 256, 64), (300, 520, 1000),
                                   (1000, 1024, 200), (17, 4096, 256), (520, 130, 264)])
@pytest.mark.parametrize("silu,add", [(0, 0), (1, 1), (1, 0), (0, 1)])
def test_matmul_f16(ctx, M, N, K, silu, add):
    rng = np.random.default_rng(M * 13 + N + K)
    a, b = half(rng, M, K, scale=0.5), half(rng, K, N, scale=0.5)
    bias = (0.1 * rng.standard_normal(N)).astype(np.float16)
    c = torch.empty(M, N, dtype=torch.float16, device="cuda")
    ctx.matmul_f16(d(a), d(b), c, M, N, K, K, N, N, d(bias), silu, add)
    ctx.sync()
    ref = O.matmul(a.astype(np.float32), b.astype(np.float32), bias.astype(np.float32), silu, add)
    err = rel_fro(h(c), ref)
    assert err <= TOL_MM and err <= TIGHT_MM, err


def test_matmul_f16_cuda_core_path_and_padding(ctx):
    # odd leading dims force the CUDA-core kernel; padding of C stays untouched
    M, N, K, lda, ldb, ldc = 37, 29, 45, 47, 31, 33
    rng = np.random.default_rng(2)
    a, b = half(rng, M, lda), half(rng, K, ldb)
    c0 = np.full((M, ldc), 7.0, np.float16)
    c = d(c0)
    ctx.matmul_f16(d(a), d(b), c, M, N, K, lda, ldb, ldc, None, 1, 0)
    ctx.sync()
    ref = O.matmul(np.ascontiguousarray(a[:, :K].astype(np.float32)),
                   np.ascontiguousarray(b[:, :N].astype(np.float32)), None, 1, 0)
    out = h(c)
    assert rel_fro(out[:, :N], ref) <= TIGHT_MM
    assert np.all(out[:, N:] == 7.0)


def test_matmul_f16_large_values_stay_finite(ctx):
    # values near the half range: fp32 accumulation, one rounding at the end
    M, N, K = 256, 256, 512
    rng = np.random.default_rng(4)
    a, b = half(rng, M, K, scale=4.0), half(rng, K, N, scale=4.0)
    c = torch.empty(M, N, dtype=torch.float16, device="cuda")
    ctx.matmul_f16(d(a), d(b), c, M, N, K, K, N, N)
    ctx.sync()
    ref = O.matmul(a.astype(np.float32), b.astype(np.float32))
    assert np.isfinite(h(c)).all() and rel_fro(h(c), ref) <= TIGHT_MM


@pytest.mark.parametrize("B,H,S,D", [(1, 2, 256, 128), (2, 1, 384, 64), (1, 1, 200, 128),
                                     (1, 2, 130, 96)])
@pytest.mark.parametrize("causal", [0, 1])
def test_attention_f16(ctx, B, H, S, D, causal):
    rng = np.random.default_rng(B * 100 + S + D + causal)
    q, k, v = (half(rng, B, H, S, D) for _ in range(3))
    o = torch.empty(B, H, S, D, dtype=torch.float16, device="cuda")
    scale = 1.0 / np.sqrt(D)
    ctx.attention_f16(d(q), d(k), d(v), o, B, H, S, S, D, scale, causal)
    ctx.sync()
    ref = O.attention_bhsd(*(t.astype(np.float32) for t in (q, k, v)), scale, causal)
    err = rel_fro(h(o), ref)
    assert err <= TOL_MM and err <= 5e-3, err


WIDE = [(1, 1), (3, 5), (7, 33), (64, 4096), (5, 4100), (3, 9000), (5, 32000), (2, 30001),
        (3, 40000)]


@pytest.mark.parametrize("rows,cols", WIDE)
def test_softmax_f16(ctx, rows, cols):
    rng = np.random.default_rng(rows + cols)
    x = half(rng, rows, cols, scale=3.0)
    y = torch.empty(rows, cols, dtype=torch.float16, device="cuda")
    ctx.softmax_f16(d(x), y, rows, cols, cols)
    ctx.sync()
    assert rel_fro(h(y), O.softmax(x.astype(np.float32))) <= TOL_ROW


@pytest.mark.parametrize("rows,cols", WIDE)
@pytest.mark.parametrize("affine", [0, 1])
def test_rmsnorm_f16(ctx, rows, cols, affine):
    rng = np.random.default_rng(rows * 3 + cols + affine)
    x = half(rng, rows, cols)
    g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float16) if affine else None
    b = (0.1 * rng.standard_normal(cols)).astype(np.float16) if affine else None
    y = torch.empty(rows, cols, dtype=torch.float16, device="cuda")
    ctx.rmsnorm_f16(d(x), y, None if g is None else d(g), None if b is None else d(b), rows, cols,
                    cols, 1e-5)
    ctx.sync()
    ref = O.rmsnorm(x.astype(np.float32), None if g is None else g.astype(np.float32),
                    None if b is None else b.astype(np.float32), 1e-5)
    assert rel_fro(h(y), ref) <= TOL_ROW


def test_casts_round_trip(ctx):
    lib = bwpp.load()
    rng = np.random.default_rng(9)
    x = (100 * rng.standard_normal(100003)).astype(np.float32)
    x[:4] = [np.inf, -np.inf, 65504.0, 1e-8]
    hx = torch.empty(x.size, dtype=torch.float16, device="cuda")
    back = torch.empty(x.size, device="cuda")
    tx = d(x)
    assert lib.bwpp_cuda_cast_f32_f16(ctx.handle, tx.data_ptr(), hx.data_ptr(), x.size) == 0
    assert lib.bwpp_cuda_cast_f16_f32(ctx.handle, hx.data_ptr(), back.data_ptr(), x.size) == 0
    ctx.sync()
    assert np.array_equal(hx.cpu().numpy(), x.astype(np.float16))  # numpy: IEEE nearest even
    assert np.array_equal(back.cpu().numpy(), x.astype(np.float16).astype(np.float32))


def test_metal_dispatch_f16_mirrors(ctx):
    lib = bwpp.load()
    rng = np.random.default_rng(6)
    M, N, K = 64, 96, 128
    a, b = half(rng, M, K, scale=0.5), half(rng, K, N, scale=0.5)
    bias = (0.1 * rng.standard_normal(N)).astype(np.float16)
    ta, tb, tbias = d(a), d(b), d(bias)
    c = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    src = b"// bwpp.meta: kernel=matmul_f16\n// bwpp.meta: epilogue=add_silu\n"
    rc = lib.bwpp_cuda_dispatch_matmul_f16(ctx.handle, ta.data_ptr(), tb.data_ptr(), c.data_ptr(),
                                           tbias.data_ptr(), bwpp.MatmulParams(M, N, K, K, N, N), src)
    ctx.sync()
    ref = O.matmul(a.astype(np.float32), b.astype(np.float32), bias.astype(np.float32), 1, 1)
    assert rc == 0 and rel_fro(h(c), ref) <= TIGHT_MM
    # #define tags select the epilogue too; kernel=none is a no-op
    c2 = torch.full((M, N), float("nan"), dtype=torch.float16, device="cuda")
    rc = lib.bwpp_cuda_dispatch_matmul_f16(ctx.handle, ta.data_ptr(), tb.data_ptr(), c2.data_ptr(),
                                           None, bwpp.MatmulParams(M, N, K, K, N, N),
                                           b"// bwpp.meta: kernel=none\n")
    ctx.sync()
    assert rc == 0 and torch.isnan(c2).all()
    src = b"// bwpp.meta: kernel=matmul_f16\n#define BWPP_EPILOGUE_SILU 1\n"
    rc = lib.bwpp_cuda_dispatch_matmul_f16(ctx.handle, ta.data_ptr(), tb.data_ptr(), c2.data_ptr(),
                                           None, bwpp.MatmulParams(M, N, K, K, N, N), src)
    ctx.sync()
    ref = O.matmul(a.astype(np.float32), b.astype(np.float32), None, 1, 0)
    assert rc == 0 and rel_fro(h(c2), ref) <= TIGHT_MM
    # rmsnorm (NULL gamma / beta) and softmax
    x = half(rng, 8, 64)
    tx = d(x)
    y = torch.empty(8, 64, dtype=torch.float16, device="cuda")
    rc = lib.bwpp_cuda_dispatch_rmsnorm_f16(ctx.handle, tx.data_ptr(), None, None, y.data_ptr(),
                                            bwpp.RmsnormParams(8, 64, 64, 1e-5),
                                            b"// bwpp.meta: aux_kernel=rmsnorm_f16\n")
    ctx.sync()
    assert rc == 0 and rel_fro(h(y), O.rmsnorm(x.astype(np.float32))) <= TOL_ROW
    rc = lib.bwpp_cuda_dispatch_softmax_f16(ctx.handle, tx.data_ptr(), y.data_ptr(),
                                            bwpp.SoftmaxParams(8, 64, 64),
                                            b"// bwpp.meta: aux_kernel=softmax_f16\n")
    ctx.sync()
    assert rc == 0 and rel_fro(h(y), O.softmax(x.astype(np.float32))) <= TOL_ROW
    # attention: 2-D unscaled (K != D: CUDA cores) and dense D = 128 (tensor cores)
    for (Mq, Nk, Kd, Dv) in ((5, 7, 24, 10), (256, 384, 128, 128)):
        q, k, v = half(rng, Mq, Kd), half(rng, Nk, Kd), half(rng, Nk, Dv)
        tq, tk, tv = d(q), d(k), d(v)
        o = torch.empty(Mq, Dv, dtype=torch.float16, device="cuda")
        rc = lib.bwpp_cuda_dispatch_attention_f16(ctx.handle, tq.data_ptr(), tk.data_ptr(),
                                                  tv.data_ptr(), o.data_ptr(),
                                                  bwpp.AttentionParams(Mq, Nk, Kd, Dv, Kd, Kd, Dv, Dv),
                                                  b"// bwpp.meta: kernel=attention_f16\n")
        ctx.sync()
        ref = O.attention2d(*(t.astype(np.float32) for t in (q, k, v)))
        assert rc == 0 and rel_fro(h(o), ref) <= 5e-3
