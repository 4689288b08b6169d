"""Norms, reduce_max and softmax on the GPU vs the CPU oracle.

Tolerances (north star): norms and reductions within 1e-5 relative Frobenius
of the fp32 oracle; argmax indices, max values and the reduce_max gradients
bit-exact.
"""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import dev, empty_f32, host, rel_fro

pytestmark = pytest.mark.gpu
TOL = 1e-5

# (rows, cols, ld): vector path, scalar path (odd cols / ld), looped path
SHAPES = [(2, 4, 4), (1, 1, 1), (5, 37, 37), (3, 1000, 1001), (64, 4096, 4096),
          (7, 4096, 4100), (33, 2048, 2048), (9, 20000, 20000), (4, 9000, 9003)]


def strided(rng, rows, cols, ld, scale=1.0):
    x = (scale * rng.standard_normal((rows, ld))).astype(np.float32)
    return x


@pytest.mark.parametrize("rows,cols,ld", SHAPES)
@pytest.mark.parametrize("affine", [False, True])
def test_rmsnorm_fwd(ctx, rows, cols, ld, affine):
    rng = np.random.default_rng(rows * 7 + cols)
    x = strided(rng, rows, cols, ld)
    g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32) if affine else None
    b = (0.1 * rng.standard_normal(cols)).astype(np.float32) if affine else None
    ref = O.rmsnorm(np.ascontiguousarray(x[:, :cols]), g, b, 1e-5)
    xd, yd = dev(x), empty_f32(rows, ld)
    ctx.rmsnorm_fwd(xd, yd, None if g is None else dev(g), None if b is None else dev(b),
                    rows, cols, ld, 1e-5)
    ctx.sync()
    y = host(yd)[:, :cols]
    assert rel_fro(y, ref) <= TOL
    if ld > cols:  # padding untouched
        assert np.isnan(host(yd)[:, cols:]).all()


def test_rmsnorm_reference_case(ctx):
    # runtime/cpu/test_metal_parity.c:186-231 (2x4 ramp, gamma = 1) and the
    # RMS ~ 1 property of runtime/cpu/test_norm.c:43-55
    x = ((np.arange(8) + 1) * np.float32(0.1)).astype(np.float32).reshape(2, 4)
    yd = empty_f32(2, 4)
    ctx.rmsnorm_fwd(dev(x), yd, dev(np.ones(4, np.float32)), None, 2, 4, 4, 1e-5)
    ctx.sync()
    y = host(yd)
    assert np.max(np.abs(y - O.rmsnorm(x, np.ones(4, np.float32)))) <= 1e-5
    assert np.all(np.abs(np.sqrt((y * y).mean(1)) - 1) <= 1e-2)


@pytest.mark.parametrize("rows,cols,ld", SHAPES)
def test_layernorm_fwd(ctx, rows, cols, ld):
    rng = np.random.default_rng(rows * 11 + cols)
    x = (3 + strided(rng, rows, cols, ld))  # offset mean exercises centring
    g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    b = (0.1 * rng.standard_normal(cols)).astype(np.float32)
    ref = O.layernorm(np.ascontiguousarray(x[:, :cols]), g, b, 1e-5)
    yd = empty_f32(rows, ld)
    ctx.layernorm_fwd(dev(x), yd, dev(g), dev(b), rows, cols, ld, 1e-5)
    ctx.sync()
    assert rel_fro(host(yd)[:, :cols], ref) <= TOL


BWD_SHAPES = [(2, 4, 4), (1, 1, 1), (300, 4096, 4096), (33, 1000, 1003), (5, 9000, 9000),
              (1000, 2048, 2048), (3, 37, 37)]


@pytest.mark.parametrize("rows,cols,ld", BWD_SHAPES)
@pytest.mark.parametrize("centered", [False, True])
def test_norm_bwd(ctx, rows, cols, ld, centered):
    rng = np.random.default_rng(rows * 13 + cols + centered)
    x = strided(rng, rows, cols, ld)
    dy = strided(rng, rows, cols, ld)
    g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
    xc, dyc = np.ascontiguousarray(x[:, :cols]), np.ascontiguousarray(dy[:, :cols])
    rdx, rdg, rdb = O.norm_bwd(xc, g, dyc, 1e-5, centered)
    dxd = empty_f32(rows, ld)
    dgd, dbd = empty_f32(cols), empty_f32(cols)
    fn = ctx.layernorm_bwd if centered else ctx.rmsnorm_bwd
    fn(dev(x), dev(g), dev(dy), dxd, dgd, dbd, rows, cols, ld, 1e-5)
    ctx.sync()
    if cols == 1:
        # one column: dx = r g (1 - xhat^2) is eps-sized, a cancellation of
        # O(r g) terms in fp32; measure the error against that term scale
        scale = np.abs(g[0] * dyc[:, 0] / np.sqrt(xc[:, 0] ** 2 + 1e-5)).max()
        assert np.abs(host(dxd)[:, :1] - rdx).max() <= TOL * scale
    else:
        assert rel_fro(host(dxd)[:, :cols], rdx) <= TOL
    assert rel_fro(host(dgd), rdg) <= TOL
    assert rel_fro(host(dbd), rdb) <= TOL


def test_norm_bwd_optional_outputs(ctx):
    rng = np.random.default_rng(1)
    x = rng.standard_normal((64, 512)).astype(np.float32)
    dy = rng.standard_normal((64, 512)).astype(np.float32)
    rdx, _, _ = O.norm_bwd(x, np.ones(512, np.float32), dy, 1e-5, False)
    dxd = empty_f32(64, 512)
    ctx.rmsnorm_bwd(dev(x), None, dev(dy), dxd, None, None, 64, 512, 512, 1e-5)
    ctx.sync()
    assert rel_fro(host(dxd), rdx) <= TOL


# ---- reduce_max ---------------------------------------------------------------

ARG_SHAPES = [(4, 4, 4), (1, 1, 1), (6, 10, 10), (5, 4097, 4099), (64, 4096, 4096),
              (3, 50000, 50000), (17, 3, 3)]


def tie_matrix(rng, rows, ld):
    x = rng.integers(-4, 4, (rows, ld)).astype(np.float32)  # dense ties
    x[0, :] = -np.inf
    if rows > 1:
        x[1, ::3] = np.nan
    return x


@pytest.mark.parametrize("rows,cols,ld", ARG_SHAPES)
@pytest.mark.parametrize("ties", [False, True])
def test_reduce_max_fwd_bwd_bit_exact(ctx, rows, cols, ld, ties):
    rng = np.random.default_rng(rows + cols)
    x = tie_matrix(rng, rows, ld) if ties else rng.standard_normal((rows, ld)).astype(np.float32)
    xc = np.ascontiguousarray(x[:, :cols])
    rmax, rarg = O.reduce_max_argmax(xc)
    md, ad = empty_f32(rows), torch.zeros(rows, dtype=torch.int32, device="cuda")
    ctx.reduce_max_fwd(dev(x), md, ad, rows, cols, ld)
    ctx.sync()
    assert np.array_equal(host(md), rmax)
    assert np.array_equal(host(ad, np.uint32), rarg)
    dy = rng.standard_normal(rows).astype(np.float32)
    dxd = empty_f32(rows, ld)
    ctx.reduce_max_bwd(ad, dev(dy), dxd, rows, cols, ld)
    ctx.sync()
    assert np.array_equal(host(dxd)[:, :cols], O.reduce_max_bwd(rarg, dy, cols))


@pytest.mark.parametrize("axis", [0, 1])
@pytest.mark.parametrize("shape", [(2, 3), (6, 10), (300, 257), (1, 1)])
def test_reduce_max_mask_and_grad_bit_exact(ctx, axis, shape):
    rows, cols = shape
    rng = np.random.default_rng(rows * cols + axis)
    x = rng.integers(-3, 3, shape).astype(np.float32)
    rm = O.reduce_max_mask(x, axis)
    md = empty_f32(rows, cols)
    ctx.reduce_max_mask(dev(x), md, rows, cols, axis)
    ctx.sync()
    assert np.array_equal(host(md), rm)
    dy = rng.standard_normal(cols if axis == 0 else rows).astype(np.float32)
    dxd = empty_f32(rows, cols)
    ctx.reduce_max_grad(md, dev(dy), dxd, rows, cols, axis)
    ctx.sync()
    assert np.array_equal(host(dxd), O.reduce_max_grad(rm, dy, axis))


@pytest.mark.parametrize("rows,cols,ld", [(2, 4, 4), (3, 50, 50), (128, 4096, 4096), (7, 333, 340)])
def test_softmax(ctx, rows, cols, ld):
    rng = np.random.default_rng(cols)
    x = (3 * rng.standard_normal((rows, ld))).astype(np.float32)
    ref = O.softmax(np.ascontiguousarray(x[:, :cols]))
    yd = empty_f32(rows, ld)
    ctx.softmax_fwd(dev(x), yd, rows, cols, ld)
    ctx.sync()
    assert rel_fro(host(yd)[:, :cols], ref) <= TOL


# ---- config 3 at full size (x 65536 x 4096 fp32) -------------------------------

def config3_inputs():
    rng = np.random.default_rng(3000)
    x = rng.standard_normal((65536, 4096), dtype=np.float32)
    g = (1 + 0.1 * rng.standard_normal(4096)).astype(np.float32)
    b = (0.1 * rng.standard_normal(4096)).astype(np.float32)
    dy = rng.standard_normal((65536, 4096), dtype=np.float32)
    return x, g, b, dy


def test_config3_full_size(ctx):
    x, g, b, dy = config3_inputs()
    R, Cc = x.shape
    xd, dyd = dev(x), dev(dy)
    yd = torch.empty_like(xd)
    # rmsnorm fwd: every row against the reference restatement
    ctx.rmsnorm_fwd(xd, yd, dev(g), dev(b), R, Cc, Cc, 1e-5)
    ctx.sync()
    assert rel_fro(host(yd), O.rmsnorm(x, g, b, 1e-5)) <= TOL
    # layernorm fwd
    ctx.layernorm_fwd(xd, yd, dev(g), dev(b), R, Cc, Cc, 1e-5)
    ctx.sync()
    assert rel_fro(host(yd), O.layernorm(x, g, b, 1e-5)) <= TOL
    # rmsnorm bwd: dx, dgamma over all 65536 rows, dbeta
    dgd, dbd = empty_f32(Cc), empty_f32(Cc)
    ctx.rmsnorm_bwd(xd, dev(g), dyd, yd, dgd, dbd, R, Cc, Cc, 1e-5)
    ctx.sync()
    rdx, rdg, rdb = O.norm_bwd(x, g, dy, 1e-5, False)
    assert rel_fro(host(yd), rdx) <= TOL
    assert rel_fro(host(dgd), rdg) <= TOL
    assert rel_fro(host(dbd), rdb) <= TOL
    # reduce_max fwd / grad, bit-exact
    md = empty_f32(R)
    ad = torch.zeros(R, dtype=torch.int32, device="cuda")
    ctx.reduce_max_fwd(xd, md, ad, R, Cc, Cc)
    ctx.sync()
    rmax, rarg = O.reduce_max_argmax(x)
    assert np.array_equal(host(md), rmax) and np.array_equal(host(ad, np.uint32), rarg)
    dyr = dy[:, 0].copy()
    ctx.reduce_max_bwd(ad, dev(dyr), yd, R, Cc, Cc)
    ctx.sync()
    out = host(yd)
    # size-independent properties of the routed gradient: one non-zero per row,
    # at the argmax, equal to dy
    assert np.array_equal(out[np.arange(R), rarg], dyr)
    assert np.count_nonzero(out) == np.count_nonzero(dyr)
    assert np.array_equal(out.sum(1, dtype=np.float64), dyr.astype(np.float64))
