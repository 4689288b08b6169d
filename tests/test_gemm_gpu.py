"""Fused matmul (+bias, +SiLU) on the GPU vs the CPU oracle.

The oracle runs on the fp32 upcast of the exact bf16 operands the kernel sees.
Tolerance (north star): relative Frobenius error <= 1e-2 against the fp32
reference.  fp32 accumulation of exact bf16 products lands near 1e-6, so a
second, tighter bound (2e-4) is asserted as a bug detector.
"""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import dev, empty_f32, host, rel_fro

pytestmark = pytest.mark.gpu
TOL = 1e-2
TIGHT = 2e-4


def operands(rng, M, N, K, lda, ldb, scale=1.0):
    a = (scale * rng.standard_normal((M, lda))).astype(np.float32)
    b = (scale * rng.standard_normal((K, ldb))).astype(np.float32)
    a16, b16 = O.f32_to_bf16(a), O.f32_to_bf16(b)
    af = np.ascontiguousarray(O.bf16_to_f32(a16)[:, :K])
    bf = np.ascontiguousarray(O.bf16_to_f32(b16)[:, :N])
    return a16, b16, af, bf


def run(ctx, a16, b16, M, N, K, lda, ldb, ldc, bias, silu, add):
    cd = empty_f32(M, ldc)
    ctx.matmul_bf16(dev(a16), dev(b16), cd, M, N, K, lda, ldb, ldc,
                    None if bias is None else dev(bias), silu, add)
    ctx.sync()
    return host(cd)


# tensor-core path: lda, ldb multiples of 8, ldc of 4
TC_SHAPES = [(128, 256, 64), (1, 8, 8), (3, 40, 24), (129, 264, 72), (300, 520, 1000),
             (256, 512, 4096), (1000, 1024, 200), (17, 11008, 256), (1024, 1024, 4096)]


@pytest.mark.parametrize("M,N,K", TC_SHAPES)
@pytest.mark.parametrize("silu,add", [(0, 0), (1, 1), (0, 1), (1, 0)])
def test_matmul_tcgen05(ctx, M, N, K, silu, add):
    rng = np.random.default_rng(M * 31 + N * 7 + K)
    a16, b16, af, bf = operands(rng, M, N, K, K, N)
    bias = rng.uniform(-0.1, 0.1, N).astype(np.float32)
    ref = O.matmul(af, bf, bias, silu, add)
    out = run(ctx, a16, b16, M, N, K, K, N, N, bias, silu, add)
    err = rel_fro(out, ref)
    assert err <= TOL and err <= TIGHT, err


def test_matmul_tcgen05_leading_dims(ctx):
    # padded rows: lda > K, ldb > N, ldc > N; the padding of C stays untouched
    M, N, K, lda, ldb, ldc = 130, 200, 136, 144, 208, 204
    rng = np.random.default_rng(5)
    a16, b16, af, bf = operands(rng, M, N, K, lda, ldb)
    bias = rng.uniform(-0.1, 0.1, N).astype(np.float32)
    out = run(ctx, a16, b16, M, N, K, lda, ldb, ldc, bias, 1, 1)
    assert rel_fro(out[:, :N], O.matmul(af, bf, bias, 1, 1)) <= TIGHT
    assert np.isnan(out[:, N:]).all()


@pytest.mark.parametrize("M,N,K,lda", [(4, 4, 4, 4), (7, 9, 5, 5), (33, 17, 0, 1)])
def test_matmul_cuda_core_fallback(ctx, M, N, K, lda):
    # shapes TMA cannot describe (pitch not a multiple of 16 B, K == 0)
    rng = np.random.default_rng(M + N + K)
    a16, b16, af, bf = operands(rng, M, N, K, max(lda, 1), N)
    bias = rng.uniform(-0.1, 0.1, N).astype(np.float32)
    out = run(ctx, a16, b16, M, N, K, max(lda, 1), N, N, bias, 1, 1)
    assert rel_fro(out, O.matmul(af, bf, bias, 1, 1)) <= TIGHT


def test_matmul_reference_case(ctx):
    # runtime/cpu/test_metal_parity.c:86-131: 4x4x4 ramp, bias 0.01*(i+1)
    a = ((np.arange(16) + 1) * np.float32(0.1)).astype(np.float32).reshape(4, 4)
    b = ((np.arange(16) + 1) * np.float32(0.05)).astype(np.float32).reshape(4, 4)
    bias = (0.01 * np.arange(1, 5)).astype(np.float32)
    a16, b16 = O.f32_to_bf16(a), O.f32_to_bf16(b)
    ref = O.matmul(O.bf16_to_f32(a16), O.bf16_to_f32(b16), bias, 1, 1)
    out = run(ctx, a16, b16, 4, 4, 4, 4, 4, 4, bias, 1, 1)
    assert np.max(np.abs(out - ref)) <= 1e-4


def test_matmul_repeated_calls_are_deterministic(ctx):
    rng = np.random.default_rng(9)
    a16, b16, _, _ = operands(rng, 512, 768, 1024, 1024, 768)
    outs = [run(ctx, a16, b16, 512, 768, 1024, 1024, 768, 768, None, 0, 0) for _ in range(3)]
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[1], outs[2])


def test_config2_full_size_sampled_rows(ctx):
    """X[8192x4096] W[4096x11008] + b, SiLU: 64 sampled rows against the oracle,
    plus size-independent properties on the full problem."""
    M, K, N = 8192, 4096, 11008
    g = torch.Generator(device="cuda").manual_seed(2000)
    x = (torch.randn(M, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    w = (torch.randn(K, N, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.rand(N, device="cuda", generator=g) * 0.2 - 0.1)
    c = torch.empty(M, N, device="cuda")
    ctx.matmul_bf16(x, w, c, M, N, K, K, N, N, b, 1, 1)
    ctx.sync()
    rows = np.unique(np.concatenate([[0, 1, 127, 128, M - 1],
                                     np.random.default_rng(1).integers(0, M, 59)]))
    xs = x[rows].float().cpu().numpy()
    wf = w.float().cpu().numpy()
    ref = O.matmul(np.ascontiguousarray(xs), np.ascontiguousarray(wf), b.cpu().numpy(), 1, 1)
    assert rel_fro(c[rows].cpu().numpy(), ref) <= TIGHT
    # size-independent properties on the full shape, no epilogue:
    # homogeneity C(2X) == 2 C(X), bit-exact (same summation order, exact
    # scaling); row permutation C(PX) == P C(X) to fp32 rounding: a row that
    # moves into a tile of the split tail has its K sum added in parts, so
    # only the order of the fp32 additions differs
    perm = torch.randperm(M, device="cuda", generator=g)
    c1, c2, c3 = (torch.empty(M, N, device="cuda") for _ in range(3))
    ctx.matmul_bf16(x, w, c1, M, N, K, K, N, N, None, 0, 0)
    ctx.matmul_bf16((x.float() * 2).to(torch.bfloat16), w, c2, M, N, K, K, N, N, None, 0, 0)
    ctx.matmul_bf16(x[perm].contiguous(), w, c3, M, N, K, K, N, N, None, 0, 0)
    ctx.sync()
    assert torch.equal(c2, 2 * c1)
    ref = c1[perm]
    assert float((c3 - ref).norm() / ref.norm()) <= 1e-6


# ---- general form: operand layouts, bf16 output, residual ---------------------

def logical(storage16, mn_major, rows, cols):
    """A operand: logical [rows=M, cols=K]; MN-major storage is [K, lda] (transposed)."""
    f = O.bf16_to_f32(storage16)
    return np.ascontiguousarray(f.T[:rows, :cols] if mn_major else f[:rows, :cols])


def logical_b(storage16, mn_major, K, N):
    """B operand: logical [K, N]; MN-major storage is [K, ldb], K-major is [N, ldb]."""
    f = O.bf16_to_f32(storage16)
    return np.ascontiguousarray(f[:K, :N] if mn_major else f[:N, :K].T)


@pytest.mark.parametrize("a_mn", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("out_bf16", [0, 1])
@pytest.mark.parametrize("M,N,K", [(256, 512, 320), (129, 264, 72), (520, 130, 1000)])
def test_gemm_ex_layouts(ctx, a_mn, b_mn, out_bf16, M, N, K):
    rng = np.random.default_rng(M + 3 * N + 7 * K + 11 * a_mn + 13 * b_mn)
    pad = lambda n: (n + 7) // 8 * 8 + 8  # leading dims > the row, multiple of 8
    # storage: A K-major [M, lda>=K] or MN-major [K, lda>=M]; B MN-major [K, ldb>=N]
    # or K-major [N, ldb>=K]
    lda = pad(M if a_mn else K)
    ldb = pad(N if b_mn else K)
    a16 = O.f32_to_bf16(rng.standard_normal((K if a_mn else M, lda)).astype(np.float32))
    b16 = O.f32_to_bf16(rng.standard_normal((K if b_mn else N, ldb)).astype(np.float32))
    A = logical(a16, a_mn, M, K)
    B = logical_b(b16, b_mn, K, N)
    bias = rng.uniform(-0.5, 0.5, N).astype(np.float32)
    resid = rng.standard_normal((M, N)).astype(np.float32)
    ref = O.matmul(A, B, bias, 1, 1) + resid
    ldc = N + 8
    if out_bf16:
        cd = torch.zeros(M, ldc, dtype=torch.int16, device="cuda")
    else:
        cd = empty_f32(M, ldc)
    ctx.gemm_ex(dev(a16), dev(b16), cd, M, N, K, lda, ldb, ldc, a_mn=a_mn, b_mn=b_mn,
                out_bf16=out_bf16, silu=1, bias=dev(bias), residual=dev(resid), ldr=N)
    ctx.sync()
    if out_bf16:
        got = O.bf16_to_f32(host(cd).view(np.uint16))[:, :N]
        err = rel_fro(got, ref)
        assert err <= TOL and err <= 5e-3, err   # bf16 output rounding ~ 2^-9
    else:
        err = rel_fro(host(cd)[:, :N], ref)
        assert err <= TOL and err <= TIGHT, err


def test_gemm_ex_accumulate_in_place(ctx):
    # residual aliasing C: C += A B (the residual add of a decoder block)
    M, N, K = 384, 768, 512
    rng = np.random.default_rng(77)
    a16 = O.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    b16 = O.f32_to_bf16(rng.standard_normal((K, N)).astype(np.float32))
    c0 = rng.standard_normal((M, N)).astype(np.float32)
    cd = dev(c0)
    ctx.gemm_ex(dev(a16), dev(b16), cd, M, N, K, K, N, N, residual=cd, ldr=N)
    ctx.sync()
    ref = O.matmul(O.bf16_to_f32(a16), O.bf16_to_f32(b16)) + c0
    assert rel_fro(host(cd), ref) <= TIGHT


@pytest.mark.parametrize("a_mn,b_mn", [(0, 0), (1, 1), (1, 0)])
def test_gemm_ex_cuda_core_layouts(ctx, a_mn, b_mn):
    # odd leading dims force the CUDA-core path; same layout semantics
    M, N, K = 37, 29, 45
    rng = np.random.default_rng(5 + a_mn + 2 * b_mn)
    lda = (M if a_mn else K) + 1
    ldb = (N if b_mn else K) + 3
    a16 = O.f32_to_bf16(rng.standard_normal((K if a_mn else M, lda)).astype(np.float32))
    b16 = O.f32_to_bf16(rng.standard_normal((K if b_mn else N, ldb)).astype(np.float32))
    A = logical(a16, a_mn, M, K)
    B = logical_b(b16, b_mn, K, N)
    cd = empty_f32(M, N)
    ctx.gemm_ex(dev(a16), dev(b16), cd, M, N, K, lda, ldb, N, a_mn=a_mn, b_mn=b_mn)
    ctx.sync()
    assert rel_fro(host(cd), O.matmul(A, B)) <= TIGHT


_SINGLE_CTA_SCRIPT = r"""
import sys
import numpy as np
sys.path[:0] = sys.argv[1:]
import bwpp, oracle as O, torch
ctx = bwpp.Ctx(0)
worst = 0.0
for (M, N, K, a_mn, b_mn) in ((300, 520, 1000, 0, 1), (1000, 1024, 200, 1, 0), (520, 130, 264, 1, 1)):
    rng = np.random.default_rng(M + N + K)
    a16 = O.f32_to_bf16(rng.standard_normal((K, M) if a_mn else (M, K)).astype(np.float32))
    b16 = O.f32_to_bf16(rng.standard_normal((K, N) if b_mn else (N, K)).astype(np.float32))
    A = O.bf16_to_f32(a16).T if a_mn else O.bf16_to_f32(a16)
    B = O.bf16_to_f32(b16) if b_mn else O.bf16_to_f32(b16).T
    c = torch.empty(M, N, device="cuda")
    ctx.gemm_ex(torch.from_numpy(a16.view(np.int16)).cuda(), torch.from_numpy(b16.view(np.int16)).cuda(), c, M, N, K,
                M if a_mn else K, N if b_mn else K, N, a_mn=a_mn, b_mn=b_mn)
    ctx.sync()
    ref = O.matmul(np.ascontiguousarray(A), np.ascontiguousarray(B))
    worst = max(worst, float(np.linalg.norm(c.cpu().numpy() - ref) / np.linalg.norm(ref)))
print("WORST", worst)
"""


def test_single_cta_kernel_with_pairs_disabled(ctx):
    """BWPP_GEMM_CTA_PAIR=0 routes every GEMM to the single-CTA kernel (the
    switch is read once per process, so this runs in a child process)."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    paths = [os.path.join(root, "bluewolf-plus-plus_b200"), os.path.join(root, "oracle")]
    env = dict(os.environ, BWPP_GEMM_CTA_PAIR="0")
    out = subprocess.run([sys.executable, "-c", _SINGLE_CTA_SCRIPT] + paths, env=env,
                         capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    worst = float(out.stdout.split("WORST")[-1])
    assert worst <= TIGHT, worst


def test_wave_tail_split_k(ctx):
    """The 8-GPU share of configs[1] (1024 x 4096 x 11008: 172 CTA-pair tiles,
    2.3 waves).  The 24-tile tail is cut into 3 K ranges run as 72 items in
    one round; the last range of each tile adds the other two from published
    partials.  Sampled rows from every 256-row block against the oracle;
    deterministic across calls."""
    M, K, N = 1024, 4096, 11008
    g = torch.Generator(device="cuda").manual_seed(77)
    x = (torch.randn(M, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    w = (torch.randn(K, N, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    b = torch.rand(N, device="cuda", generator=g) * 0.2 - 0.1
    c = torch.empty(M, N, device="cuda")
    ctx.matmul_bf16(x, w, c, M, N, K, K, N, N, b, 1, 1)
    ctx.sync()
    rows = np.unique(np.concatenate([[0, 255, 256, 511, 512, 767, 768, 1023],
                                     np.random.default_rng(3).integers(0, M, 40)]))
    ref = O.matmul(np.ascontiguousarray(x[rows].float().cpu().numpy()),
                   np.ascontiguousarray(w.float().cpu().numpy()), b.cpu().numpy(), 1, 1)
    assert rel_fro(c[rows].cpu().numpy(), ref) <= TIGHT
    # deterministic across calls
    c2 = torch.empty_like(c)
    ctx.matmul_bf16(x, w, c2, M, N, K, K, N, N, b, 1, 1)
    ctx.sync()
    assert torch.equal(c, c2)


def test_split_tail_with_half_the_sms_held_by_another_stream(ctx):
    """The split tail must not need all of its CTAs resident at once: here
    another stream holds half of the SMs (full shared memory each) for 2.5 s,
    longer than the kernels' 2 s wait limit, while the 1024 x 4096 x 11008
    GEMM runs on the rest.  Parts that start early count themselves in and
    leave their partials; the parts that start after the hold ends finish
    the tiles.  Status OK, and bit-identical to the same GEMM run alone (the
    partial sums fold in part order whichever part finishes a tile)."""
    import bwpp
    M, K, N = 1024, 4096, 11008
    g = torch.Generator(device="cuda").manual_seed(78)
    x = (torch.randn(M, K, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    w = (torch.randn(K, N, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    b = torch.rand(N, device="cuda", generator=g) * 0.2 - 0.1
    alone = torch.empty(M, N, device="cuda")
    ctx.matmul_bf16(x, w, alone, M, N, K, K, N, N, b, 1, 1)
    ctx.sync()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    other = torch.cuda.Stream()
    torch.cuda.synchronize()
    held = torch.empty(M, N, device="cuda")
    rc = ctx.lib.bwpp_cuda_selftest_occupy(ctx.handle, other.cuda_stream, sms // 2, 200 * 1024, 2500)
    assert rc == bwpp.OK
    ctx.matmul_bf16(x, w, held, M, N, K, K, N, N, b, 1, 1)
    ctx.sync()  # raises on BWPP_CUDA_ERR_TIMEOUT
    torch.cuda.synchronize()
    assert torch.equal(held, alone)
    rows = np.arange(0, M, 37)
    ref = O.matmul(np.ascontiguousarray(x[rows].float().cpu().numpy()),
                   np.ascontiguousarray(w.float().cpu().numpy()), b.cpu().numpy(), 1, 1)
    assert rel_fro(held[rows].cpu().numpy(), ref) <= TIGHT


# Split-tail cases: (M, N, K, a_mn, b_mn, out_bf16, residual)
#  - 2 tiles: each tile's 128 K blocks cut into 8 parts (7 partials per owner)
#  - M <= 128 (single-CTA kernel): 8 tiles cut into 8 parts each
#  - ragged M, N and K (last K block partly out of bounds), all four layouts
SK_CASES = [(256, 512, 8192, 0, 1, 0, 0), (128, 2048, 4096, 0, 1, 0, 0),
            (700, 1000, 3000, 0, 1, 0, 1), (384, 640, 3000, 1, 0, 1, 1),
            (520, 264, 2048, 1, 1, 0, 0), (300, 777, 1560, 0, 0, 1, 0)]


@pytest.mark.parametrize("M,N,K,a_mn,b_mn,out_bf16,residual", SK_CASES)
def test_split_tail_tiles(ctx, M, N, K, a_mn, b_mn, out_bf16, residual):
    rng = np.random.default_rng(M + 5 * N + 3 * K + a_mn + 2 * b_mn)
    lda = (M if a_mn else K) + 8 - (M if a_mn else K) % 8
    ldb = (N if b_mn else K) + 8 - (N if b_mn else K) % 8
    a16 = O.f32_to_bf16(rng.standard_normal((K if a_mn else M, lda)).astype(np.float32))
    b16 = O.f32_to_bf16(rng.standard_normal((K if b_mn else N, ldb)).astype(np.float32))
    A = logical(a16, a_mn, M, K)
    B = logical_b(b16, b_mn, K, N)
    bias = rng.uniform(-0.5, 0.5, N).astype(np.float32)
    res = rng.standard_normal((M, N)).astype(np.float32) if residual else None
    ref = O.matmul(A, B, bias, 1, 1) + (res if residual else 0)
    kw = dict(a_mn=a_mn, b_mn=b_mn, out_bf16=out_bf16, silu=1, bias=dev(bias))
    if residual:
        kw.update(residual=dev(res), ldr=N)
    outs = []
    for _ in range(2):
        if out_bf16:
            cd = torch.zeros(M, N, dtype=torch.int16, device="cuda")
        else:
            cd = empty_f32(M, N)
        ctx.gemm_ex(dev(a16), dev(b16), cd, M, N, K, lda, ldb, N, **kw)
        ctx.sync()
        outs.append(host(cd))
    assert np.array_equal(outs[0], outs[1])  # the partial sums add in a fixed order
    if out_bf16:
        got = O.bf16_to_f32(outs[0].view(np.uint16))
        err = rel_fro(got, ref)
        assert err <= TOL and err <= 5e-3, err
    else:
        err = rel_fro(outs[0], ref)
        assert err <= TOL and err <= TIGHT, err


def test_wave_tail_in_half_tiles(ctx):
    """K below 8 blocks of 64 is not cut into K parts; the tail keeps N
    halves: 2 x 4 tiles of 256 x 256, fewer than half the CTA pairs, each
    run as two N halves."""
    M, N, K = 512, 1024, 256
    rng = np.random.default_rng(21)
    a16, b16, af, bf = operands(rng, M, N, K, K, N)
    bias = rng.uniform(-0.1, 0.1, N).astype(np.float32)
    out = run(ctx, a16, b16, M, N, K, K, N, N, bias, 1, 1)
    assert rel_fro(out, O.matmul(af, bf, bias, 1, 1)) <= TIGHT


def test_whole_tile_tail_small_k(ctx):
    """K below 8 blocks and a tail wider than half the CTA pairs (5 x 9 = 45
    tiles): the tail runs as whole tiles, neither halved nor cut in K."""
    M, N, K = 1100, 2100, 200
    rng = np.random.default_rng(23)
    a16, b16, af, bf = operands(rng, M, N, K, K, N)
    bias = rng.uniform(-0.1, 0.1, N).astype(np.float32)
    out = run(ctx, a16, b16, M, N, K, K, N, N, bias, 1, 1)
    assert rel_fro(out, O.matmul(af, bf, bias, 1, 1)) <= TIGHT


@pytest.mark.parametrize("out_bf16", [0, 1])
def test_split_tiles_with_residual_and_16bit_out(ctx, out_bf16):
    # 2 x 4 tiles of 256 x 256 with 16 K blocks: each tile is cut into 4 K
    # parts; the owner adds the residual (aliasing C) once
    M, N, K = 512, 1024, 1024
    rng = np.random.default_rng(8 + out_bf16)
    a16 = O.f32_to_bf16(rng.standard_normal((M, K)).astype(np.float32))
    b16 = O.f32_to_bf16(rng.standard_normal((K, N)).astype(np.float32))
    res = rng.standard_normal((M, N)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, N).astype(np.float32)
    ref = O.matmul(O.bf16_to_f32(a16), O.bf16_to_f32(b16), bias, 1, 1) + res
    if out_bf16:
        c = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        ctx.gemm_ex(dev(a16), dev(b16), c, M, N, K, K, N, N, out_bf16=1, silu=1, bias=dev(bias),
                    residual=dev(res), ldr=N)
        ctx.sync()
        assert rel_fro(c.float().cpu().numpy(), ref) <= 5e-3
    else:
        cd = dev(res)  # residual aliases C: C = silu(A B + bias) + C
        ctx.gemm_ex(dev(a16), dev(b16), cd, M, N, K, K, N, N, silu=1, bias=dev(bias), residual=cd,
                    ldr=N)
        ctx.sync()
        assert rel_fro(host(cd), ref) <= TIGHT
