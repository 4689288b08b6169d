"""Drop-in mirrors: the exact CPU-reference signatures (host or device buffers)
and the Metal dispatch calls with bwpp.meta source text, vs the oracle."""
import ctypes as C

import numpy as np
import pytest
import torch

import bwpp
import oracle as O
from conftest import dev, empty_f32, host, rel_fro

pytestmark = pytest.mark.gpu


def ramp(r, c, s):
    return ((np.arange(r * c) + 1) * np.float32(s)).astype(np.float32).reshape(r, c)


@pytest.mark.parametrize("where", ["host", "device"])
def test_cpu_mirror_matmul(ctx, where):
    # bwpp_cpu_matmul_f32 signature; fp32 inputs rounded to bf16 on the device
    for M, N, K in [(4, 4, 4), (70, 130, 90), (256, 256, 256)]:
        rng = np.random.default_rng(M)
        a = rng.standard_normal((M, K)).astype(np.float32)
        b = rng.standard_normal((K, N)).astype(np.float32)
        bias = rng.uniform(-0.1, 0.1, N).astype(np.float32)
        ref = O.matmul(O.round_bf16(a), O.round_bf16(b), bias, 1, 1)
        if where == "host":
            c = np.zeros((M, N), np.float32)
            bwpp.matmul_f32(a, b, c, M, N, K, K, N, N, bias, 1, 1)
        else:
            cd = empty_f32(M, N)
            bwpp.matmul_f32(dev(a), dev(b), cd, M, N, K, K, N, N, dev(bias), 1, 1)
            c = host(cd)
        assert rel_fro(c, ref) <= 2e-4


def test_cpu_mirror_matmul_strided_host():
    M, N, K, lda, ldb, ldc = 9, 7, 5, 11, 13, 10
    rng = np.random.default_rng(2)
    a = rng.standard_normal((M, lda)).astype(np.float32)
    b = rng.standard_normal((K, ldb)).astype(np.float32)
    c = np.full((M, ldc), 7.0, np.float32)
    bwpp.matmul_f32(a, b, c, M, N, K, lda, ldb, ldc, None, 0, 0)
    ref = O.matmul(O.round_bf16(np.ascontiguousarray(a[:, :K])), O.round_bf16(np.ascontiguousarray(b[:, :N])))
    assert rel_fro(c[:, :N], ref) <= 2e-4
    assert (c[:, N:] == 7.0).all()


@pytest.mark.parametrize("M,N,K,pad,bias_on", [(2500, 2100, 300, 3, 1), (1100, 5000, 160, 0, 0),
                                               (4096, 900, 96, 5, 1)])
def test_cpu_mirror_matmul_host_pipelined(M, N, K, pad, bias_on):
    """Host A, B and C large enough to be cut into row and column chunks:
    uploads, GEMMs of each L-shaped region and strided downloads overlap on
    three streams.  Every element of C (and none of its padding) is written."""
    lda, ldb, ldc = K + pad, N + pad, N + 2 * pad
    rng = np.random.default_rng(M + N)
    a = rng.standard_normal((M, lda)).astype(np.float32)
    b = rng.standard_normal((K, ldb)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, N).astype(np.float32) if bias_on else None
    c = np.full((M, ldc), 7.0, np.float32)
    ref = O.matmul(O.round_bf16(np.ascontiguousarray(a[:, :K])),
                   O.round_bf16(np.ascontiguousarray(b[:, :N])), bias, bias_on, bias_on)
    for _ in range(2):  # the second call reuses the copy streams and events
        bwpp.matmul_f32(a, b, c, M, N, K, lda, ldb, ldc, bias, bias_on, bias_on)
        assert rel_fro(c[:, :N], ref) <= 2e-4
        assert (c[:, N:] == 7.0).all()
        c[:, :N] = np.nan


@pytest.mark.parametrize("where", ["host", "device"])
def test_cpu_mirror_rows(ctx, where):
    rng = np.random.default_rng(4)
    x = rng.standard_normal((6, 300)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(300)).astype(np.float32)
    put = (lambda a: a) if where == "host" else dev
    get = (lambda a: a) if where == "host" else host
    y = np.zeros_like(x) if where == "host" else empty_f32(6, 300)
    bwpp.rmsnorm_f32(put(x), y, put(g), None, 6, 300, 300, 1e-5)
    assert rel_fro(get(y), O.rmsnorm(x, g, None, 1e-5)) <= 1e-5
    y = np.zeros_like(x) if where == "host" else empty_f32(6, 300)
    bwpp.softmax_f32(put(x), y, 6, 300, 300)
    assert rel_fro(get(y), O.softmax(x)) <= 1e-5
    xt = rng.integers(-2, 2, (5, 9)).astype(np.float32)
    for axis in (0, 1):
        m = np.zeros_like(xt) if where == "host" else empty_f32(5, 9)
        bwpp.reduce_max_mask_f32(put(xt), m, 5, 9, axis)
        assert np.array_equal(get(m), O.reduce_max_mask(xt, axis))
        dy = rng.standard_normal(9 if axis == 0 else 5).astype(np.float32)
        dx = np.zeros_like(xt) if where == "host" else empty_f32(5, 9)
        bwpp.reduce_max_grad_f32(put(O.reduce_max_mask(xt, axis)), put(dy), dx, 5, 9, axis)
        assert np.array_equal(get(dx), O.reduce_max_grad(O.reduce_max_mask(xt, axis), dy, axis))


def test_cpu_mirror_reference_known_answers():
    # runtime/cpu/test_reduce_max.c and test_norm.c, through the CUDA mirrors
    x = np.arange(6, dtype=np.float32).reshape(2, 3)
    m = np.zeros_like(x)
    bwpp.reduce_max_mask_f32(x, m, 2, 3, 1)
    assert np.array_equal(m, np.array([[0, 0, 1], [0, 0, 1]], np.float32))
    dx = np.zeros_like(x)
    bwpp.reduce_max_grad_f32(m, np.array([1, 2], np.float32), dx, 2, 3, 1)
    assert np.array_equal(dx, np.array([[0, 0, 1], [0, 0, 2]], np.float32))
    xs = ramp(2, 4, 0.1)
    y = np.zeros_like(xs)
    bwpp.softmax_f32(xs, y, 2, 4, 4)
    assert np.all(np.abs(y.sum(1) - 1) <= 1e-3)


def test_cpu_mirror_null_is_silent_noop():
    c = np.full((2, 2), 3.0, np.float32)
    bwpp.load().bwpp_cuda_matmul_f32(None, None, c.ctypes.data, 2, 2, 2, 2, 2, 2, None, 0, 0)
    assert bwpp.load().bwpp_cuda_last_status() == bwpp.OK
    assert (c == 3.0).all()


META_MM = """// bwpp.meta: kernel=matmul_f16
// bwpp.meta: epilogue=add_silu
"""


def test_metal_dispatch_mirrors(ctx):
    lib = bwpp.load()
    rng = np.random.default_rng(6)
    M, N, K = 64, 96, 128
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((K, N)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, N).astype(np.float32)
    a16, b16 = O.f32_to_bf16(a), O.f32_to_bf16(b)
    ta, tb, tbias = dev(a16), dev(b16), dev(bias)  # kept alive while the kernels run
    cd = empty_f32(M, N)
    p = bwpp.MatmulParams(M, N, K, K, N, N)
    rc = lib.bwpp_cuda_dispatch_matmul(ctx.handle, ta.data_ptr(), tb.data_ptr(),
                                       cd.data_ptr(), tbias.data_ptr(), p, META_MM.encode())
    assert rc == 0
    ctx.sync()
    ref = O.matmul(O.bf16_to_f32(a16), O.bf16_to_f32(b16), bias, 1, 1)
    assert rel_fro(host(cd), ref) <= 2e-4
    # kernel=none: the call is a no-op (runtime/metal/dispatch_stub.m:74-76)
    cd2 = empty_f32(M, N)
    rc = lib.bwpp_cuda_dispatch_matmul(ctx.handle, ta.data_ptr(), tb.data_ptr(),
                                       cd2.data_ptr(), None, p, b"// bwpp.meta: kernel=none\n")
    ctx.sync()
    assert rc == 0 and torch.isnan(cd2).all()
    # rmsnorm with NULL gamma / beta acts as ones / zeros
    x = rng.standard_normal((8, 64)).astype(np.float32)
    tx = dev(x)
    yd = empty_f32(8, 64)
    rc = lib.bwpp_cuda_dispatch_rmsnorm(ctx.handle, tx.data_ptr(), None, None, yd.data_ptr(),
                                        bwpp.RmsnormParams(8, 64, 64, 1e-5),
                                        b"// bwpp.meta: aux_kernel=rmsnorm_f16\n")
    ctx.sync()
    assert rc == 0 and rel_fro(host(yd), O.rmsnorm(x)) <= 1e-5
    xs = rng.standard_normal((4, 33)).astype(np.float32)
    txs = dev(xs)
    yd = empty_f32(4, 33)
    rc = lib.bwpp_cuda_dispatch_softmax(ctx.handle, txs.data_ptr(), yd.data_ptr(),
                                        bwpp.SoftmaxParams(4, 33, 33),
                                        b"// bwpp.meta: aux_kernel=softmax_f16\n")
    ctx.sync()
    assert rc == 0 and rel_fro(host(yd), O.softmax(xs)) <= 1e-5
    # attention: the reference's 2-D unscaled form with K != D
    q = rng.standard_normal((5, 24)).astype(np.float32)
    k = rng.standard_normal((7, 24)).astype(np.float32)
    v = rng.standard_normal((7, 10)).astype(np.float32)
    q16, k16, v16 = (O.f32_to_bf16(t) for t in (q, k, v))
    tq, tk, tv = dev(q16), dev(k16), dev(v16)
    od = empty_f32(5, 10)
    rc = lib.bwpp_cuda_dispatch_attention(ctx.handle, tq.data_ptr(), tk.data_ptr(),
                                          tv.data_ptr(), od.data_ptr(),
                                          bwpp.AttentionParams(5, 7, 24, 10, 24, 24, 10, 10),
                                          b"// bwpp.meta: kernel=attention_f16\n")
    ctx.sync()
    ref = O.attention2d(*(O.bf16_to_f32(t) for t in (q16, k16, v16)))
    assert rc == 0 and rel_fro(host(od), ref) <= 2e-3


def test_arena_one_allocation(ctx):
    lib = bwpp.load()
    arena = bwpp.Arena()
    assert lib.bwpp_cuda_arena_init(C.byref(arena), 1 << 20, 0) == 1
    p1 = lib.bwpp_cuda_arena_alloc(C.byref(arena), 100, 256)
    p2 = lib.bwpp_cuda_arena_alloc(C.byref(arena), 100, 256)
    assert p1 % 256 == 0 and p2 - p1 == 256
    assert lib.bwpp_cuda_arena_alloc(C.byref(arena), 1 << 20, 16) is None  # full -> NULL
    assert lib.bwpp_cuda_arena_alloc(C.byref(arena), 8, 3) is None          # align not 2^k
    lib.bwpp_cuda_arena_reset(C.byref(arena))
    assert lib.bwpp_cuda_arena_alloc(C.byref(arena), 8, 0) == p1
    lib.bwpp_cuda_arena_destroy(C.byref(arena))
    assert arena.capacity == 0


def test_device_timeout_status_is_reported(ctx):
    """A kernel's bounded wait that expires comes back as BWPP_CUDA_ERR_TIMEOUT
    from bwpp_cuda_sync, and the context keeps working afterwards."""
    lib = bwpp.load()
    assert lib.bwpp_cuda_selftest_wait_timeout(ctx.handle, 0) == bwpp.ERR_ARG
    assert lib.bwpp_cuda_selftest_wait_timeout(ctx.handle, 50) == bwpp.OK
    assert lib.bwpp_cuda_sync(ctx.handle) == bwpp.ERR_TIMEOUT
    assert lib.bwpp_cuda_sync(ctx.handle) == bwpp.OK  # cleared
    x = np.ones((2, 8), np.float32)
    yd = empty_f32(2, 8)
    ctx.rmsnorm_fwd(dev(x), yd, None, None, 2, 8, 8, 0.0)
    ctx.sync()
    assert np.allclose(host(yd), 1.0)


@pytest.mark.parametrize("mode", [["--cuda"], []])
def test_c_bench_twin_schema(tmp_path, mode):
    """bwpp_bench_cuda keeps the reference bench's CLI and JSON keys
    (bench/bench_cpu.c:45-63,142-158), so bench/bench_regress.py can read it."""
    import json
    import subprocess
    exe = bwpp.PKG_ROOT + "/bench/bwpp_bench_cuda"
    out = tmp_path / "b.json"
    r = subprocess.run([exe, "--iters", "3", "--m", "128", "--n", "256", "--k", "64", "--rows", "64",
                        "--cols", "512", "--json", str(out)] + mode, capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    d = json.loads(out.read_text())
    assert set(d["matmul"]) == {"M", "N", "K", "iters", "time_s", "gflops"}
    assert d["matmul"]["gflops"] > 0 and d["softmax"]["time_s"] > 0 and d["rmsnorm"]["rows"] == 64
