"""Autodiff-internal graph ops on the GPU (silu_grad, softmax_grad,
reduce_sum, broadcast) against the CPU oracle.

The reference emits these ops from its backward rules
(compiler/graph_ir.c:1414-1470, 1709-1733, 1791-1796) but has no kernel for
them, so parity is against the oracle's float64 restatement (itself checked
against torch autograd in test_oracle.py).  Tolerance: relative Frobenius
<= 1e-5 (north star bound for reductions and row operations); broadcast is
bit-exact.
"""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import dev, host, rel_fro

pytestmark = pytest.mark.gpu
TOL = 1e-5

SHAPES = [(1, 1), (3, 5), (7, 33), (64, 4096), (5, 4100), (17, 9000), (300, 257)]


def randn(rng, *shape, scale=1.0):
    return (scale * rng.standard_normal(shape)).astype(np.float32)


@pytest.mark.parametrize("n", [1, 3, 4, 1000, 1 << 20, (1 << 20) + 3])
def test_silu_grad(ctx, n):
    rng = np.random.default_rng(n)
    x, dy = randn(rng, n, scale=4.0), randn(rng, n)
    dx = torch.empty(n, device="cuda")
    ctx.silu_grad(dev(x), dev(dy), dx, n)
    ctx.sync()
    assert rel_fro(host(dx), O.silu_grad(x, dy)) <= TOL


def test_silu_grad_extremes_and_in_place(ctx):
    x = np.array([-1e4, -100, -88.8, -20, -1e-8, 0, 1e-8, 20, 88.8, 100, 1e4, 3.0], np.float32)
    dy = np.linspace(-2, 2, x.size).astype(np.float32)
    d = dev(dy)
    ctx.silu_grad(dev(x), d, d, x.size)  # in place over dy
    ctx.sync()
    ref = O.silu_grad(x, dy)
    np.testing.assert_allclose(host(d), ref, rtol=1e-5, atol=1e-30)


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_softmax_grad(ctx, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    x = randn(rng, rows, cols, scale=3.0)
    y = (np.exp(x - x.max(1, keepdims=True))
         / np.exp(x - x.max(1, keepdims=True)).sum(1, keepdims=True)).astype(np.float32)
    dy = randn(rng, rows, cols)
    dx = torch.empty(rows, cols, device="cuda")
    ctx.softmax_grad(dev(y), dev(dy), dx, rows, cols, cols)
    ctx.sync()
    ref = O.softmax_grad(y, dy)
    assert rel_fro(host(dx), ref) <= TOL


def test_softmax_grad_padded_rows_and_alias(ctx):
    rows, cols, ld = 9, 130, 136
    rng = np.random.default_rng(3)
    y = np.abs(randn(rng, rows, ld))
    dy = randn(rng, rows, ld)
    d = dev(dy)
    ctx.softmax_grad(dev(y), d, d, rows, cols, ld)  # dx aliases dy
    ctx.sync()
    out = host(d)
    ref = O.softmax_grad(np.ascontiguousarray(y[:, :cols]), np.ascontiguousarray(dy[:, :cols]))
    assert rel_fro(out[:, :cols], ref) <= TOL
    assert np.array_equal(out[:, cols:], dy[:, cols:])  # padding untouched


@pytest.mark.parametrize("rows,cols", SHAPES + [(65536, 64), (1, 100000)])
@pytest.mark.parametrize("axis", [0, 1])
def test_reduce_sum(ctx, rows, cols, axis):
    rng = np.random.default_rng(rows + cols + axis)
    x = randn(rng, rows, cols)
    out = torch.empty(rows if axis == 1 else cols, device="cuda")
    ctx.reduce_sum(dev(x), out, rows, cols, cols, axis)
    ctx.sync()
    assert rel_fro(host(out), O.reduce_sum(x, axis)) <= TOL


def test_reduce_sum_empty_and_deterministic(ctx):
    out = torch.full((5,), 7.0, device="cuda")
    ctx.reduce_sum(dev(np.zeros((5, 1), np.float32)), out, 5, 0, 1, 1)
    ctx.sync()
    assert torch.equal(out, torch.zeros(5, device="cuda"))
    rng = np.random.default_rng(11)
    x = dev(randn(rng, 4096, 1024))
    a, b = torch.empty(1024, device="cuda"), torch.empty(1024, device="cuda")
    ctx.reduce_sum(x, a, 4096, 1024, 1024, 0)
    ctx.reduce_sum(x, b, 4096, 1024, 1024, 0)
    ctx.sync()
    assert torch.equal(a, b)


@pytest.mark.parametrize("rows,cols", SHAPES)
@pytest.mark.parametrize("axis", [0, 1])
def test_broadcast_bit_exact(ctx, rows, cols, axis):
    rng = np.random.default_rng(rows * cols + axis)
    src = randn(rng, rows if axis == 1 else cols)
    dst = torch.empty(rows, cols, device="cuda")
    ctx.broadcast(dev(src), dst, rows, cols, cols, axis)
    ctx.sync()
    assert np.array_equal(host(dst), O.broadcast(src, rows, cols, axis))


def test_reduce_sum_broadcast_is_the_gradient_pair(ctx):
    """<reduce_sum(x), g> == <x, broadcast(g)> (adjoint pair), float64 check."""
    rng = np.random.default_rng(5)
    rows, cols = 513, 1027
    x, g0, g1 = randn(rng, rows, cols), randn(rng, cols), randn(rng, rows)
    for axis, g in ((0, g0), (1, g1)):
        s = torch.empty(g.size, device="cuda")
        bx = torch.empty(rows, cols, device="cuda")
        ctx.reduce_sum(dev(x), s, rows, cols, cols, axis)
        ctx.broadcast(dev(g), bx, rows, cols, cols, axis)
        ctx.sync()
        lhs = float(host(s).astype(np.float64) @ g.astype(np.float64))
        rhs = float((x.astype(np.float64) * host(bx).astype(np.float64)).sum())
        assert abs(lhs - rhs) <= 1e-4 * (abs(rhs) + np.sqrt(rows * cols))
