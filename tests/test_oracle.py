"""Pins the CPU oracle (oracle/bwpp_oracle.c) to the reference.

1. Golden fixtures made by the reference's own library (tests/golden/) must be
   reproduced bit-for-bit.
2. When oracle/_ref (the reference compiled from its sources) is present, the
   oracle must equal it bit-for-bit on fresh seeded inputs.
3. The assertions of the reference's own tests hold for the oracle
   (runtime/cpu/test_norm.c, test_reduce_max.c, test_metal_parity.c).
4. The extensions the reference lacks are checked against float64 numpy /
   torch autograd (parity unpinned by the reference).
"""
import os

import numpy as np
import pytest

import oracle as O
from conftest import rel_fro

GOLD = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_golden.npz"))


def same(a, b):
    return np.array_equal(np.asarray(a), np.asarray(b))


# ---- 1. golden fixtures ----------------------------------------------------

@pytest.mark.parametrize("add", [0, 1])
@pytest.mark.parametrize("silu", [0, 1])
def test_golden_matmul_ramp(add, silu):
    out = O.matmul(GOLD["mm4_a"], GOLD["mm4_b"], GOLD["mm4_bias"], silu, add)
    assert same(out, GOLD[f"mm4_out_add{add}_silu{silu}"])


def test_golden_bench_matmul_256():
    # bench/bench_cpu.c:82-83 ramp fill, 256^3
    i = np.arange(256 * 256, dtype=np.float64).reshape(256, 256)
    a = ((i + 1).astype(np.float32) * np.float32(0.01)).astype(np.float32)
    b = ((i + 1).astype(np.float32) * np.float32(0.02)).astype(np.float32)
    out = O.matmul(a, b, np.zeros(256, np.float32), 0, 0)
    assert same(out, GOLD["bench_mm_out"])


def test_golden_softmax_rmsnorm_attention():
    assert same(O.softmax(GOLD["sm_x"]), GOLD["sm_out"])
    assert same(O.rmsnorm(GOLD["rms_x"], GOLD["rms_gamma"], None, 1e-5), GOLD["rms_out"])
    assert same(O.attention2d(GOLD["att_q"], GOLD["att_k"], GOLD["att_v"]), GOLD["att_out"])


def test_golden_reduce_max():
    x = GOLD["rmax_x"]
    m1 = O.reduce_max_mask(x, 1)
    assert same(m1, GOLD["rmax_mask1"])
    assert same(O.reduce_max_grad(m1, GOLD["rmax_dy"], 1), GOLD["rmax_grad1"])
    m0 = O.reduce_max_mask(x, 0)
    assert same(m0, GOLD["rmax_mask0"])
    assert same(O.reduce_max_grad(m0, np.array([1, 2, 3], np.float32), 0), GOLD["rmax_grad0"])


def test_golden_random_cases():
    assert same(O.matmul(GOLD["rmm_a"], GOLD["rmm_b"], GOLD["rmm_bias"], 1, 1), GOLD["rmm_out"])
    assert same(O.rmsnorm(GOLD["rrms_x"], GOLD["rrms_gamma"], GOLD["rrms_beta"], 1e-5), GOLD["rrms_out"])
    assert same(O.softmax(GOLD["rsm_x"]), GOLD["rsm_out"])
    assert same(O.attention2d(GOLD["ratt_q"], GOLD["ratt_k"], GOLD["ratt_v"]), GOLD["ratt_out"])
    x = GOLD["rrmax_x"]
    for axis, dy in ((0, GOLD["rrmax_dyc"]), (1, GOLD["rrmax_dyr"])):
        m = O.reduce_max_mask(x, axis)
        assert same(m, GOLD[f"rrmax_mask{axis}"])
        assert same(O.reduce_max_grad(m, dy, axis), GOLD[f"rrmax_grad{axis}"])


# ---- 2. live comparison with the reference library -------------------------

ref = O.ref_lib()
needs_ref = pytest.mark.skipif(ref is None, reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("shape", [(1, 1, 1), (3, 5, 7), (33, 65, 17), (64, 40, 96)])
def test_live_matmul_bit_exact(shape):
    M, K, N = shape
    rng = np.random.default_rng(M * 1000 + N)
    a = rng.standard_normal((M, K)).astype(np.float32)
    b = rng.standard_normal((K, N)).astype(np.float32)
    bias = rng.uniform(-1, 1, N).astype(np.float32)
    for add in (0, 1):
        for silu in (0, 1):
            assert same(O.matmul(a, b, bias, silu, add), O.matmul(a, b, bias, silu, add, lib=ref))


@needs_ref
def test_live_rows_bit_exact():
    rng = np.random.default_rng(7)
    x = (2 * rng.standard_normal((13, 300))).astype(np.float32)
    g = rng.standard_normal(300).astype(np.float32)
    bt = rng.standard_normal(300).astype(np.float32)
    assert same(O.softmax(x), O.softmax(x, lib=ref))
    for gamma, beta in ((None, None), (g, None), (g, bt)):
        assert same(O.rmsnorm(x, gamma, beta, 1e-5), O.rmsnorm(x, gamma, beta, 1e-5, lib=ref))
    xt = rng.integers(-2, 2, (9, 31)).astype(np.float32)
    for axis in (0, 1):
        assert same(O.reduce_max_mask(xt, axis), O.reduce_max_mask(xt, axis, lib=ref))


@needs_ref
def test_live_attention_bit_exact():
    rng = np.random.default_rng(11)
    q = rng.standard_normal((5, 24)).astype(np.float32)
    k = rng.standard_normal((19, 24)).astype(np.float32)
    v = rng.standard_normal((19, 10)).astype(np.float32)
    assert same(O.attention2d(q, k, v), O.attention2d(q, k, v, lib=ref))


# ---- 3. the reference tests' own assertions ---------------------------------

def test_reference_test_norm_assertions():
    # runtime/cpu/test_norm.c:31-55: softmax rows sum to 1 (1e-3), rmsnorm RMS 1 (1e-2)
    x = GOLD["sm_x"]
    assert np.all(np.abs(O.softmax(x).sum(1) - 1) <= 1e-3)
    z = O.rmsnorm(x, np.ones(4, np.float32), None, 1e-5)
    assert np.all(np.abs(np.sqrt((z * z).mean(1)) - 1) <= 1e-2)


def test_reference_test_reduce_max_assertions():
    # runtime/cpu/test_reduce_max.c:13-55: one-hot at the last column, dx = dy[r] there
    x = np.arange(6, dtype=np.float32).reshape(2, 3)
    m = O.reduce_max_mask(x, 1)
    assert same(m, np.array([[0, 0, 1], [0, 0, 1]], np.float32))
    dx = O.reduce_max_grad(m, np.array([1, 2], np.float32), 1)
    assert same(dx, np.array([[0, 0, 1], [0, 0, 2]], np.float32))


def test_reference_parity_restatements():
    # runtime/cpu/test_metal_parity.c: the inline restatements agree with the
    # library to 1e-4 (matmul) / 1e-5 (softmax, rmsnorm, attention)
    a, b, bias = GOLD["mm4_a"], GOLD["mm4_b"], GOLD["mm4_bias"]
    ref = a.astype(np.float64) @ b.astype(np.float64) + bias
    ref = ref / (1 + np.exp(-ref))
    assert np.max(np.abs(O.matmul(a, b, bias, 1, 1) - ref)) <= 1e-4
    q, k, v = GOLD["att_q"], GOLD["att_k"], GOLD["att_v"]
    s = q.astype(np.float64) @ k.T
    p = np.exp(s - s.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    assert np.max(np.abs(O.attention2d(q, k, v) - p @ v)) <= 1e-5


# ---- 4. extensions (unpinned by the reference) ------------------------------

def np_norm_fwd(x, gamma, beta, eps, centered):
    x = x.astype(np.float64)
    mu = x.mean(1, keepdims=True) if centered else 0.0
    r = 1 / np.sqrt(((x - mu) ** 2).mean(1, keepdims=True) + eps)
    return (x - mu) * r * gamma + beta


@pytest.mark.parametrize("centered", [False, True])
def test_norm_extensions_vs_torch_autograd(centered):
    import torch
    rng = np.random.default_rng(3)
    x = rng.standard_normal((7, 129)).astype(np.float32)
    g = (1 + 0.1 * rng.standard_normal(129)).astype(np.float32)
    bt = (0.1 * rng.standard_normal(129)).astype(np.float32)
    dy = rng.standard_normal((7, 129)).astype(np.float32)
    if centered:
        y = O.layernorm(x, g, bt, 1e-5)
        assert rel_fro(y, np_norm_fwd(x, g, bt, 1e-5, True)) < 1e-6
    tx = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    tg = torch.tensor(g, dtype=torch.float64, requires_grad=True)
    tb = torch.tensor(bt, dtype=torch.float64, requires_grad=True)
    mu = tx.mean(1, keepdim=True) if centered else 0.0
    ty = (tx - mu) * torch.rsqrt(((tx - mu) ** 2).mean(1, keepdim=True) + 1e-5) * tg + tb
    ty.backward(torch.tensor(dy, dtype=torch.float64))
    dx, dg, db = O.norm_bwd(x, g, dy, 1e-5, centered)
    assert rel_fro(dx, tx.grad.numpy()) < 1e-6
    assert rel_fro(dg, tg.grad.numpy()) < 1e-6
    assert rel_fro(db, tb.grad.numpy()) < 1e-6


def test_argmax_first_index_and_edges():
    x = np.array([[1, 3, 3, 0],            # tie -> first
                  [-np.inf] * 4,           # nothing > -inf -> 0
                  [np.nan, 2, np.nan, 2],  # NaN skipped, tie -> 1
                  [5, -1, -7, 5]], np.float32)
    mx, am = O.reduce_max_argmax(x)
    assert list(am) == [1, 0, 1, 0]
    assert mx[0] == 3 and mx[1] == -np.inf and mx[2] == 2 and mx[3] == 5
    dy = np.array([1, 2, 3, 4], np.float32)
    dx = O.reduce_max_bwd(am, dy, 4)
    exp = np.zeros((4, 4), np.float32)
    exp[np.arange(4), am] = dy
    assert same(dx, exp)
    # on tie-free rows the argmax-routed gradient equals the reference's mask form
    rng = np.random.default_rng(5)
    xr = rng.standard_normal((8, 33)).astype(np.float32)
    _, a2 = O.reduce_max_argmax(xr)
    assert same(O.reduce_max_bwd(a2, dy.repeat(2), 33),
                O.reduce_max_grad(O.reduce_max_mask(xr, 1), dy.repeat(2), 1))


@pytest.mark.parametrize("causal", [0, 1])
def test_attention_bhsd_vs_float64(causal):
    rng = np.random.default_rng(9)
    B, H, S, D = 2, 3, 33, 16
    q, k, v = (rng.standard_normal((B, H, S, D)).astype(np.float32) for _ in range(3))
    scale = 1 / np.sqrt(D)
    s = np.einsum("bhmd,bhnd->bhmn", q.astype(np.float64), k) * scale
    if causal:
        s = np.where(np.tril(np.ones((S, S), bool)), s, -np.inf)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    ref = np.einsum("bhmn,bhnd->bhmd", p, v)
    slow = O.attention_bhsd(q, k, v, scale, causal, fast=False)
    fast = O.attention_bhsd(q, k, v, scale, causal, fast=True)
    assert rel_fro(slow, ref) < 1e-5
    assert rel_fro(fast, ref) < 1e-5
    part = O.attention_bhsd(q, k, v, scale, causal, rows=(5, 9))
    assert same(part[:, :, 5:9], fast[:, :, 5:9]) and not part[:, :, :5].any()


def test_bf16_round_trip():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.4e38, 1e-40, np.inf], np.float32)
    h = O.f32_to_bf16(x)
    # 1 + 2^-8 is a tie between 1 and 1 + 2^-7: nearest even keeps 1.0
    assert h[0] == 0x3F80 and h[1] == 0x3F80 and h[2] == 0x3F82
    assert O.bf16_to_f32(h)[3] == -2.5 and np.isinf(O.bf16_to_f32(h)[4])
    assert np.isnan(O.round_bf16(np.array([np.nan], np.float32)))[0]


def test_autodiff_ops_vs_torch_autograd():
    """silu_grad / softmax_grad against float64 torch autograd; reduce_sum and
    broadcast against numpy (the reference has rules, no kernels, for these)."""
    import torch
    rng = np.random.default_rng(17)
    x = (3 * rng.standard_normal((37, 53))).astype(np.float32)
    dy = rng.standard_normal((37, 53)).astype(np.float32)
    xt = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    torch.nn.functional.silu(xt).backward(torch.tensor(dy, dtype=torch.float64))
    np.testing.assert_allclose(O.silu_grad(x, dy), xt.grad.numpy(), rtol=1e-6, atol=1e-7)
    xt = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    yt = torch.softmax(xt, -1)
    yt.backward(torch.tensor(dy, dtype=torch.float64))
    y = yt.detach().numpy().astype(np.float32)
    np.testing.assert_allclose(O.softmax_grad(y, dy), xt.grad.numpy(), rtol=1e-5, atol=1e-7)
    for axis in (0, 1):
        np.testing.assert_allclose(O.reduce_sum(x, axis), x.astype(np.float64).sum(axis),
                                   rtol=1e-6, atol=1e-6)
    col = rng.standard_normal(53).astype(np.float32)
    row = rng.standard_normal(37).astype(np.float32)
    assert np.array_equal(O.broadcast(col, 37, 53, 0), np.broadcast_to(col, (37, 53)))
    assert np.array_equal(O.broadcast(row, 37, 53, 1), np.broadcast_to(row[:, None], (37, 53)))
