"""Training path on the GPU: attention forward with log-sum-exp and attention
backward, then the whole tiny_model step (BASELINE configs[4] at reduced
size), against float64 torch autograd on the CPU.

The reference has no backward kernels and no model step (parity unpinned by
the reference); the checker is a float64 restatement of the same math.  For
the model step the restatement rounds to bf16 at the points where the GPU
stores bf16 (straight-through in the backward), so the comparison isolates
kernel error from the chosen storage precision.
Tolerances: relative Frobenius <= 1e-2 for attention (north star bound for
contractions); <= 3e-2 for the composed gradients of the whole step (every
layer's backward rounds its activation gradients to bf16 once more).
"""
import math

import numpy as np
import pytest
import torch

import bwpp
import oracle as O
from conftest import rel_fro

pytestmark = pytest.mark.gpu


def bf16(t):
    return t.to(torch.bfloat16)


def ref_attention(q, k, v, scale, causal):
    s = (q @ k.transpose(-1, -2)) * scale
    if causal:
        S = s.shape[-1]
        s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool), 1), float("-inf"))
    return torch.softmax(s, -1) @ v, torch.logsumexp(s, -1) / math.log(2.0)


def heads(t, B, S, H, D=128):  # token-major [B*S, H*D] -> [B, H, S, D]
    return t.reshape(B, S, H, D).permute(0, 2, 1, 3)


# (1, 2, 1024): 8 query / key tiles, so every pipeline barrier wraps its
# phase several times; (1, 1, 200): a ragged last tile (zero-filled rows);
# (2, 2, 200): the ragged tile's dK / dV store stops at its own sequence
@pytest.mark.parametrize("B,H,S", [(2, 2, 256), (1, 3, 384), (2, 1, 128), (1, 2, 1024), (1, 1, 200),
                                   (2, 2, 200)])
@pytest.mark.parametrize("causal", [1, 0])
def test_attention_fwd_lse_and_bwd(ctx, B, H, S, causal):
    D, lib = 128, bwpp.load()
    g = torch.Generator(device="cuda").manual_seed(B * 100 + S + causal)
    T, HD = B * S, H * 128
    q, k, v, do = (bf16(torch.randn(T, HD, device="cuda", generator=g)) for _ in range(4))
    o = torch.empty(T, HD, dtype=torch.bfloat16, device="cuda")
    lse = torch.empty(B * H * S, device="cuda")
    scale = 1.0 / math.sqrt(D)
    ctx.check(lib.bwpp_cuda_attention_fwd_lse_bf16(ctx.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                                   HD, B, H, S, scale, causal, o.data_ptr(), HD,
                                                   lse.data_ptr()), "fwd_lse")
    dq, dk, dv = (torch.empty(T, HD, dtype=torch.bfloat16, device="cuda") for _ in range(3))
    ctx.check(lib.bwpp_cuda_attention_bwd_bf16(ctx.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), HD,
                                               o.data_ptr(), HD, do.data_ptr(), HD, lse.data_ptr(), B, H,
                                               S, scale, causal, dq.data_ptr(), dk.data_ptr(),
                                               dv.data_ptr(), HD), "bwd")
    ctx.sync()
    qf, kf, vf, dof = (heads(t.double().cpu(), B, S, H).requires_grad_(True) for t in (q, k, v, do))
    ro, rlse = ref_attention(qf, kf, vf, scale, causal)
    ro.backward(dof.detach())
    got_o = heads(o.double().cpu(), B, S, H)
    assert rel_fro(got_o.numpy(), ro.detach().numpy()) <= 1e-2
    assert np.abs(lse.cpu().numpy().reshape(B, H, S) - rlse.detach().numpy()).max() <= 2e-2
    for got, ref in ((dq, qf.grad), (dk, kf.grad), (dv, vf.grad)):
        err = rel_fro(heads(got.double().cpu(), B, S, H).numpy(), ref.numpy())
        assert err <= 1e-2, err


def test_attention_bwd_rejects_unaligned_outputs(ctx):
    """Output bases off a 16-byte boundary are refused (the backward kernels
    store 16-byte vectors and bulk tiles)."""
    lib, B, H, S = bwpp.load(), 1, 1, 128
    T, HD = B * S, H * 128
    x = torch.zeros(T * HD + 8, dtype=torch.bfloat16, device="cuda")
    lse = torch.zeros(B * H * S, device="cuda")
    p = x.data_ptr()
    rc = lib.bwpp_cuda_attention_bwd_bf16(ctx.handle, p, p, p, HD, p, HD, p, HD, lse.data_ptr(), B, H, S,
                                          0.1, 1, p, p + 8, p, HD)
    assert rc == bwpp.ERR_UNSUPPORTED


# ---- tiny_model step -----------------------------------------------------------

def split_params(flat, L, D, F):
    out, off = [], 0
    for _ in range(L):
        layer = {}
        for name, n, shape in (("g1", D, (D,)), ("wqkv", 3 * D * D, (D, 3 * D)), ("wo", D * D, (D, D)),
                               ("g2", D, (D,)), ("w13", 2 * F * D, (D, 2 * F)), ("w2", F * D, (F, D))):
            layer[name] = flat[off:off + n].reshape(shape)
            off += n
        out.append(layer)
    return out


def st_bf16(t):
    """Round to bf16 in the forward, identity in the backward."""
    return t + (t.to(torch.bfloat16).to(t.dtype) - t).detach()


def ref_model_step(flat, x, tgt, L, D, H, F, B, S, eps):
    params = flat.clone().requires_grad_(True)
    P = split_params(params, L, D, F)
    h = x.clone()
    scale = 1.0 / math.sqrt(128)

    def rms(u, gam):
        return u * torch.rsqrt((u * u).mean(-1, keepdim=True) + eps) * gam

    for p in P:
        w = {k_: st_bf16(v_) if v_.dim() == 2 else v_ for k_, v_ in p.items()}
        n1 = st_bf16(rms(h, w["g1"]))
        qkv = st_bf16(n1 @ w["wqkv"])
        q, k, v = (heads(qkv[:, i * D:(i + 1) * D], B, S, H) for i in range(3))
        o, _ = ref_attention(q, k, v, scale, True)
        o = st_bf16(o.permute(0, 2, 1, 3).reshape(B * S, D))
        h = h + o @ w["wo"]
        n2 = st_bf16(rms(h, w["g2"]))
        gu = st_bf16(n2 @ w["w13"])
        a = st_bf16(torch.nn.functional.silu(gu[:, :F]) * gu[:, F:])
        h = h + a @ w["w2"]
    loss = ((h - tgt) ** 2).mean()
    loss.backward()
    return float(loss.detach()), params.grad


def test_tiny_model_step_vs_float64():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    L, D, H, F, B, S, eps = 2, 256, 2, 512, 2, 256, 1e-5
    ctx = bwpp.Ctx(0)
    model = bwpp.TinyModel(ctx, L, D, H, F, B, S, eps, seed=3)
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(B * S, D, device="cuda", generator=g)
    tgt = torch.randn(B * S, D, device="cuda", generator=g)
    params = torch.empty(model.count, device="cuda")
    grads = torch.empty(model.count, device="cuda")
    model.get(params, None)
    loss = torch.empty(1, device="cuda")
    model.step(x, tgt, lr=0.0, loss_out=loss)
    model.get(None, grads)
    rloss, rgrad = ref_model_step(params.double().cpu(), x.double().cpu(), tgt.double().cpu(),
                                  L, D, H, F, B, S, eps)
    assert abs(float(loss) - rloss) <= 2e-3 * abs(rloss)
    gp = split_params(grads.double().cpu(), L, D, F)
    rp = split_params(rgrad, L, D, F)
    for l in range(L):
        for name in gp[l]:
            err = rel_fro(gp[l][name].numpy(), rp[l][name].numpy())
            assert err <= 3e-2, (l, name, err)
    # SGD: params' = params - lr * grads (one GPU: the mean is the gradient)
    before = params.clone()
    model.step(x, tgt, lr=0.1, loss_out=loss)
    model.get(params, grads)
    assert torch.allclose(params, before - 0.1 * grads, rtol=0, atol=1e-6)
    # the step is deterministic
    g1 = grads.clone()
    model.set_params(before)
    model.step(x, tgt, lr=0.0, loss_out=loss)
    model.get(None, grads)
    assert torch.equal(grads, g1)
    model.close()
    ctx.close()


def test_gradient_of_concatenated_batch_is_mean_of_per_batch_gradients():
    """The identity the data-parallel step rests on, on one GPU: the gradient
    of the MSE loss over a batch of 2B sequences equals the mean of the
    gradients over its two halves of B.  Per-sequence work is identical in
    both runs (the MSE scale halves exactly), so the two sides differ only
    by fp32 reassociation of the sums over tokens (dW, dgamma).  A step that
    dropped or double-counted a half would be off by O(1)."""
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    L, D, H, F, B, S, eps = 2, 256, 2, 512, 2, 256, 1e-5
    ctx = bwpp.Ctx(0)
    half = bwpp.TinyModel(ctx, L, D, H, F, B, S, eps, seed=3)
    full = bwpp.TinyModel(ctx, L, D, H, F, 2 * B, S, eps, seed=3)
    g = torch.Generator(device="cuda").manual_seed(21)
    x = torch.randn(2 * B * S, D, device="cuda", generator=g)
    tgt = torch.randn(2 * B * S, D, device="cuda", generator=g)
    parts = []
    for i in range(2):
        rows = slice(i * B * S, (i + 1) * B * S)
        half.step(x[rows].contiguous(), tgt[rows].contiguous(), lr=0.0)
        gr = torch.empty(half.count, device="cuda")
        half.get(None, gr)
        parts.append(gr)
    full.step(x, tgt, lr=0.0)
    g_cat = torch.empty(full.count, device="cuda")
    full.get(None, g_cat)
    mean = (parts[0].double() + parts[1].double()) / 2
    err = float(torch.linalg.norm(g_cat.double() - mean) / torch.linalg.norm(mean))
    assert err <= 1e-4, err
    # and one SGD step on the full batch applies lr times that gradient (to
    # within one fp32 rounding of the weights, |w| <= ~0.1)
    p0 = torch.empty(full.count, device="cuda")
    full.get(p0, None)
    full.step(x, tgt, lr=0.1)
    p1 = torch.empty(full.count, device="cuda")
    full.get(p1, None)
    assert torch.allclose(p1, p0 - 0.1 * g_cat, rtol=0, atol=1e-6)
    assert float((p1 - p0).abs().max()) > 1e-5  # the step moved the weights
    half.close()
    full.close()
    ctx.close()


def _ref_attention_dev(q, k, v, scale):
    s = (q @ k.transpose(-1, -2)) * scale
    S = s.shape[-1]
    s = s.masked_fill(torch.triu(torch.ones(S, S, dtype=torch.bool, device=s.device), 1), float("-inf"))
    return torch.softmax(s, -1) @ v


def ref_model_grads_chunked(flat, x, tgt, L, D, H, F, B, S, eps, chunk):
    """float64 restatement of the step (same bf16 rounding points as
    ref_model_step) on the GPU, over `chunk` sequences at a time: the loss is
    the mean over all B sequences, so each chunk's backward adds its share of
    the parameter gradient; returns (loss, d params, d x)."""
    params = flat.clone().requires_grad_(True)
    n_total = float(B * S * D)
    scale = 1.0 / math.sqrt(128)
    loss = 0.0
    dx = torch.empty_like(x)

    def rms(u, gam):
        return u * torch.rsqrt((u * u).mean(-1, keepdim=True) + eps) * gam

    for b0 in range(0, B, chunk):
        cb = min(chunk, B - b0)
        rows = slice(b0 * S, (b0 + cb) * S)
        xb = x[rows].clone().requires_grad_(True)
        P = split_params(params, L, D, F)
        h = xb
        for p in P:
            w = {k_: st_bf16(v_) if v_.dim() == 2 else v_ for k_, v_ in p.items()}
            n1 = st_bf16(rms(h, w["g1"]))
            qkv = st_bf16(n1 @ w["wqkv"])
            q, k, v = (heads(qkv[:, i * D:(i + 1) * D], cb, S, H) for i in range(3))
            o = st_bf16(_ref_attention_dev(q, k, v, scale).permute(0, 2, 1, 3).reshape(cb * S, D))
            h = h + o @ w["wo"]
            n2 = st_bf16(rms(h, w["g2"]))
            gu = st_bf16(n2 @ w["w13"])
            a = st_bf16(torch.nn.functional.silu(gu[:, :F]) * gu[:, F:])
            h = h + a @ w["w2"]
        part = ((h - tgt[rows]) ** 2).sum() / n_total
        part.backward()
        loss += float(part.detach())
        dx[rows] = xb.grad
        del h, part, xb
    return loss, params.grad, dx


def test_tiny_model_step_config5_shape_vs_float64():
    """configs[4] at its own shape (2 layers, d_model 2048, 16 x 128 heads,
    causal, gated MLP 5632, seq 2048, batch 16): the loss, every layer's
    weight gradients, the norm-gain gradients and 40 sampled rows of
    d loss / d x against the float64 restatement (run on the GPU in chunks
    of 4 sequences).  Tolerances as at the reduced shape."""
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    L, D, H, F, B, S, eps = 2, 2048, 16, 5632, 16, 2048, 1e-5
    ctx = bwpp.Ctx(0)
    model = bwpp.TinyModel(ctx, L, D, H, F, B, S, eps, seed=1)
    g = torch.Generator(device="cuda").manual_seed(5000)
    x = torch.randn(B * S, D, device="cuda", generator=g)
    tgt = torch.randn(B * S, D, device="cuda", generator=g)
    params = torch.empty(model.count, device="cuda")
    grads = torch.empty(model.count, device="cuda")
    dx = torch.empty(B * S, D, device="cuda")
    loss = torch.empty(1, device="cuda")
    model.get(params, None)
    model.step(x, tgt, lr=0.0, loss_out=loss)
    model.get(None, grads)
    model.input_grad(dx)
    model.close()
    ctx.close()
    rloss, rgrad, rdx = ref_model_grads_chunked(params.double(), x.double(), tgt.double(),
                                                L, D, H, F, B, S, eps, chunk=4)
    assert abs(float(loss) - rloss) <= 2e-3 * abs(rloss), (float(loss), rloss)
    gp = split_params(grads.double(), L, D, F)
    rp = split_params(rgrad, L, D, F)
    for l in range(L):
        for name in gp[l]:
            a, b = gp[l][name], rp[l][name]
            err = float(torch.linalg.norm(a - b) / torch.linalg.norm(b))
            assert err <= 3e-2, (l, name, err)
    rows = torch.tensor(sorted({0, 1, S - 1, S, B * S - 1} |
                               set(np.random.default_rng(9).integers(0, B * S, 35).tolist())),
                        device="cuda")
    a, b = dx[rows].double(), rdx[rows]
    err = float(torch.linalg.norm(a - b) / torch.linalg.norm(b))
    assert err <= 3e-2, err
