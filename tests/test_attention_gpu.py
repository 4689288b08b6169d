"""Attention O = softmax(scale * Q K^T [causal]) V on the GPU vs the CPU oracle.

The oracle (runtime/cpu/bwpp_cpu_ref.c:92-144 restated, q pre-scaled, causal
rows cut at n <= m) runs on the fp32 upcast of the exact bf16 inputs.
Tolerance (north star): relative Frobenius error <= 1e-2; a tighter 2e-3 bound
is asserted as a bug detector (P is rounded to bf16 before the PV product on
the tensor-core path).
"""
import numpy as np
import pytest
import torch

import oracle as O
from conftest import dev, empty_f32, host, rel_fro

pytestmark = pytest.mark.gpu
TOL = 1e-2
TIGHT = 2e-3


def qkv(rng, B, H, Sq, Skv, D):
    q = rng.standard_normal((B, H, Sq, D)).astype(np.float32)
    k = rng.standard_normal((B, H, Skv, D)).astype(np.float32)
    v = rng.standard_normal((B, H, Skv, D)).astype(np.float32)
    return [O.f32_to_bf16(t) for t in (q, k, v)]


def run(ctx, q16, k16, v16, B, H, Sq, Skv, D, scale, causal):
    od = empty_f32(B, H, Sq, D)
    ctx.attention_bf16(dev(q16), dev(k16), dev(v16), od, B, H, Sq, Skv, D, scale, causal)
    ctx.sync()
    return host(od)


SHAPES = [(1, 1, 128, 128, 128), (2, 3, 33, 33, 64), (1, 2, 300, 300, 128), (1, 1, 1, 1, 128),
          (2, 2, 256, 512, 64), (1, 1, 257, 129, 128), (1, 1, 64, 64, 32), (1, 2, 40, 40, 96)]


@pytest.mark.parametrize("B,H,Sq,Skv,D", SHAPES)
@pytest.mark.parametrize("causal", [0, 1])
def test_attention(ctx, B, H, Sq, Skv, D, causal):
    if causal and Sq > Skv:
        pytest.skip("causal needs Sq <= Skv")
    rng = np.random.default_rng(B * 100 + Sq + D + causal)
    q16, k16, v16 = qkv(rng, B, H, Sq, Skv, D)
    scale = 1.0 / np.sqrt(D)
    ref = O.attention_bhsd(*(O.bf16_to_f32(t) for t in (q16, k16, v16)), scale, causal)
    out = run(ctx, q16, k16, v16, B, H, Sq, Skv, D, scale, causal)
    err = rel_fro(out, ref)
    assert err <= TOL and err <= TIGHT, err


def test_attention_reference_case(ctx):
    # runtime/cpu/test_metal_parity.c:233-302: M=2 N=3 K=4 D=5 ramps, no scale/mask
    ramp = lambda r, c, s: ((np.arange(r * c) + 1) * np.float32(s)).astype(np.float32).reshape(r, c)
    q, k, v = ramp(2, 4, 0.03), ramp(3, 4, 0.04), ramp(3, 5, 0.02)
    qb, kb, vb = (O.round_bf16(t) for t in (q, k, v))
    ref = O.attention2d(qb, kb, vb)
    import bwpp
    o = np.zeros((2, 5), np.float32)
    bwpp.attention_f32(q, k, v, o, 2, 3, 4, 5, 4, 4, 5, 5)
    assert np.max(np.abs(o - ref)) <= 2e-3


def test_config4_sampled_rows(ctx):
    """B=8 H=32 S=4096 D=128, causal and not: 8 query rows of every (b,h)
    (including 0, 1 and S-1) against the oracle."""
    B, H, S, D = 8, 32, 4096, 128
    g = torch.Generator(device="cuda").manual_seed(4000)
    q, k, v = (torch.randn(B, H, S, D, device="cuda", generator=g).to(torch.bfloat16)
               for _ in range(3))
    scale = 1.0 / np.sqrt(D)
    rows = [0, 1, 777, 1500, 2049, 3000, 4000, S - 1]
    qf, kf, vf = (t.float().cpu().numpy() for t in (q, k, v))
    for causal in (0, 1):
        o = torch.empty(B, H, S, D, device="cuda")
        ctx.attention_bf16(q, k, v, o, B, H, S, S, D, scale, causal)
        ctx.sync()
        got = o[:, :, rows].cpu().numpy()
        ref = np.stack([O.attention_bhsd(qf, kf, vf, scale, causal, rows=(r, r + 1))[:, :, r]
                        for r in rows], axis=2)
        err = rel_fro(got, ref)
        assert err <= TOL and err <= TIGHT, (causal, err)



# Non-causal launches whose last round of items (256 query rows of one head
# each, one CTA per SM) would be at most half full run those items in a second
# launch, as two halves over the key blocks merged in global memory: 160 items
# leave 12 for it.  Checked against the oracle, with ragged Sq / Skv (the
# second half holds the masked key edge) and in the half ABI, run to run
# bit-identical (the merge is in half order), and against the same heads in a
# launch of exactly 148 items (no split).
SPLIT_SHAPES = [(40, 1024, 1024, 128), (40, 1000, 777, 128), (40, 1024, 1024, 64)]


@pytest.mark.parametrize("BH,Sq,Skv,D", SPLIT_SHAPES)
def test_attention_split_tail(ctx, BH, Sq, Skv, D):
    pairs = -(-Sq // 256)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    if not (pairs * BH > sms and 0 < (pairs * BH) % sms <= sms // 2):
        pytest.skip(f"{pairs * BH} items leave no split tail on {sms} SMs")
    rng = np.random.default_rng(Sq + Skv + D)
    q16, k16, v16 = qkv(rng, 1, BH, Sq, Skv, D)
    scale = 1.0 / np.sqrt(D)
    out = run(ctx, q16, k16, v16, 1, BH, Sq, Skv, D, scale, 0)
    again = run(ctx, q16, k16, v16, 1, BH, Sq, Skv, D, scale, 0)
    assert np.array_equal(out.view(np.uint32), again.view(np.uint32))
    ref = O.attention_bhsd(*(O.bf16_to_f32(t) for t in (q16, k16, v16)), scale, 0)
    err = rel_fro(out, ref)
    assert err <= TOL and err <= TIGHT, err
    # the halves round P to bf16 against their own running maxima, so a
    # launch without the split agrees to about bf16 over the key sum
    nh = sms // pairs
    tail = run(ctx, q16[:, -nh:], k16[:, -nh:], v16[:, -nh:], 1, nh, Sq, Skv, D, scale, 0)
    assert rel_fro(out[:, -nh:], tail) <= 1e-3


def test_attention_split_tail_half_abi(ctx):
    """The half ABI (f16 in, f16 out) through the same split tail."""
    BH, S, D = 40, 1024, 128
    rng = np.random.default_rng(77)
    q, k, v = (rng.standard_normal((BH, S, D)).astype(np.float16) for _ in range(3))
    qd, kd, vd = (torch.from_numpy(t).cuda() for t in (q, k, v))
    od = torch.empty(BH, S, D, dtype=torch.float16, device="cuda")
    ctx.attention_f16(qd, kd, vd, od, 1, BH, S, S, D, 1.0 / np.sqrt(D), 0)
    ctx.sync()
    ref = O.attention_bhsd(q.astype(np.float32)[None], k.astype(np.float32)[None],
                           v.astype(np.float32)[None], 1.0 / np.sqrt(D), 0)[0]
    assert rel_fro(od.float().cpu().numpy(), ref) <= TOL
