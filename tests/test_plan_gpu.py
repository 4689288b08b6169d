"""Launch-plan executor on the GPU: graphs built by the reference compiler
(its own --dot / --grad-dot / --mem-plan dumps of the reference examples,
tests/golden/plans/) run end to end on the CUDA kernels and are compared with
a CPU composition of the oracle's restatements of runtime/cpu/bwpp_cpu_ref.c
(forward) or float64 torch autograd (gradient graphs, whose rules
compiler/graph_ir.c:1529-1796 states but no reference kernel runs).

Every value is stored as the graph declares it (f16), so intermediate
results are rounded to half; tolerances: relative Frobenius <= 1e-2 for one
contraction, <= 3e-2 for a composed model (as the training-step test)."""
import os

import numpy as np
import pytest
import torch

import bwpp
import oracle as O
from conftest import rel_fro

pytestmark = pytest.mark.gpu
PLANS = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "plans")


def dump(name, ext=".dot"):
    with open(os.path.join(PLANS, name + ext)) as f:
        return f.read()


def half(rng, *shape, scale=1.0):
    return (scale * rng.standard_normal(shape)).astype(np.float16)


def f32(a):
    return np.asarray(a, np.float32)


def run(ctx, name, dims, inputs, grad=False, options=None, mem=True):
    plan = bwpp.Plan(ctx, dump(name, ".grad.dot" if grad else ".dot"),
                     dump(name, ".mem.txt") if mem and not grad else None, dims, options)
    for key, arr in inputs.items():
        plan.bind(key, torch.from_numpy(np.ascontiguousarray(arr)).cuda())
    plan.run()
    ctx.sync()
    outs = {v["id"]: plan.tensor(v["id"]).float().cpu().numpy() for v in plan.values() if v["output"]}
    launches = plan.launches
    plan.close()
    return outs, launches


@pytest.mark.parametrize("fuse", [1, 0])
def test_matmul_add_silu(ctx, fuse):
    M, K, N = 200, 256, 384
    rng = np.random.default_rng(1)
    a, b, bias = half(rng, M, K, scale=0.5), half(rng, K, N, scale=0.5), half(rng, N, scale=0.1)
    outs, launches = run(ctx, "matmul_add_silu", dict(M=M, K=K, N=N), {"a": a, "b": b, "bias": bias},
                         options=f"fuse={fuse}")
    ref = O.matmul(f32(a), f32(b), f32(bias), 1, 1)
    (out,) = outs.values()
    assert rel_fro(out, ref) <= 2e-3
    assert launches == (1 if fuse else 3)


def test_matmul_add_reshaped_bias(ctx):
    M, K, N = 129, 136, 264
    rng = np.random.default_rng(2)
    a, b, bias = half(rng, M, K), half(rng, K, N), half(rng, N)
    outs, launches = run(ctx, "matmul_add_bias_reshape", dict(M=M, K=K, N=N), {"a": a, "b": b, "bias": bias})
    (out,) = outs.values()
    assert rel_fro(out, O.matmul(f32(a), f32(b), f32(bias), 0, 1)) <= 2e-3 and launches == 1


def test_norms_graph(ctx):
    B, N = 96, 512
    rng = np.random.default_rng(3)
    x, w = half(rng, B, N, scale=0.2), half(rng, N, N, scale=0.2)
    gamma = (1 + 0.1 * rng.standard_normal(N)).astype(np.float16)
    outs, _ = run(ctx, "norms", dict(B=B, N=N), {"x": x, "w": w, "gamma": gamma})
    y = O.matmul(f32(x), f32(w)).astype(np.float16)  # the graph stores y as f16
    ref = O.rmsnorm(O.softmax(f32(y)), f32(gamma), None, 1e-5)
    (out,) = outs.values()
    assert rel_fro(out, ref) <= 1e-2


@pytest.mark.parametrize("D", [64, 128, 96])
def test_attention_graph_rank4(ctx, D):
    B, H, T = 2, 3, 256
    rng = np.random.default_rng(D)
    q, k, v = (half(rng, B, H, T, D, scale=0.3) for _ in range(3))
    outs, launches = run(ctx, "attention", dict(B=B, H=H, T=T, D=D), {"q": q, "k": k, "v": v})
    ref = O.attention_bhsd(f32(q), f32(k), f32(v), 1.0, 0)  # the graph is unscaled, unmasked
    (out,) = outs.values()
    assert out.shape == (B, H, T, D) and launches == 1
    assert rel_fro(out, ref) <= 1e-2


def tiny_forward_ref(p, eps=1e-5):
    """fp32 composition of examples/tiny_model.bwpp with the oracle restatements."""
    def block(x, pre):
        n1 = O.rmsnorm(x, p["g1" + pre], None, eps)
        q, k, v = (O.matmul(n1, p[w + pre]) for w in ("wq", "wk", "wv"))
        s = O.softmax(O.matmul(q, np.ascontiguousarray(k.T)))
        a = O.matmul(O.matmul(s, v), p["wo" + pre])
        x1 = x + a
        n2 = O.rmsnorm(x1, p["g2" + pre], None, eps)
        h = O.matmul(n2, p["w1" + pre])
        h = h / (1 + np.exp(-h))
        return x1 + O.matmul(h.astype(np.float32), p["w2" + pre])
    h1 = block(p["x"], "1")
    h2 = block(h1, "2")
    return O.softmax(O.matmul(h2, p["wcls"]))


@pytest.mark.parametrize("fuse", [1, 0])
def test_tiny_model_forward(ctx, fuse):
    T, D, H, V = 256, 128, 256, 512
    rng = np.random.default_rng(7)
    p = {"x": half(rng, T, D)}
    for pre in ("1", "2"):
        for w in ("wq", "wk", "wv", "wo"):
            p[w + pre] = half(rng, D, D, scale=D ** -0.5)
        p["w1" + pre] = half(rng, D, H, scale=D ** -0.5)
        p["w2" + pre] = half(rng, H, D, scale=H ** -0.5)
        p["g1" + pre] = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
        p["g2" + pre] = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    p["wcls"] = half(rng, D, V, scale=D ** -0.5)
    outs, launches = run(ctx, "tiny_model", dict(T=T, D=D, H=H, V=V), p, options=f"fuse={fuse}")
    ref = tiny_forward_ref({k: f32(v) for k, v in p.items()})
    (out,) = outs.values()
    assert out.shape == (T, V)
    assert rel_fro(out, ref) <= 3e-2
    assert launches == (20 if fuse else 32)


def test_grad_graph_matmul_add_silu(ctx):
    """Gradient graph: inputs a, b, bias, y = a@b + bias (activation) and the
    output gradient; outputs dbias, da, db."""
    M, K, N = 192, 128, 256
    rng = np.random.default_rng(11)
    a, b, bias = half(rng, M, K, scale=0.5), half(rng, K, N, scale=0.5), half(rng, N, scale=0.1)
    y = (f32(a) @ f32(b) + f32(bias)).astype(np.float16)
    dout = half(rng, M, N)
    plan = bwpp.Plan(ctx, dump("matmul_add_silu", ".grad.dot"), None, dict(M=M, K=K, N=N))
    seed = [v["id"] for v in plan.values() if v["input"] and v["id"] not in
            (plan.id("a"), plan.id("b"), plan.id("bias"), plan.id("y"))]
    assert len(seed) == 1
    keep = []
    for key, arr in (("a", a), ("b", b), ("bias", bias), ("y", y), (seed[0], dout)):
        t = torch.from_numpy(arr).cuda()
        keep.append(t)
        plan.bind(key, t)
    plan.run()
    ctx.sync()
    got = {v["shape"]: plan.tensor(v["id"]).double().cpu() for v in plan.values() if v["output"]}
    at, bt, bit = (torch.tensor(f32(u), dtype=torch.float64, requires_grad=True) for u in (a, b, bias))
    yt = at @ bt + bit
    torch.nn.functional.silu(yt).backward(torch.tensor(f32(dout), dtype=torch.float64))
    assert rel_fro(got[(N,)].numpy(), bit.grad.numpy()) <= 1e-2
    assert rel_fro(got[(M, K)].numpy(), at.grad.numpy()) <= 1e-2
    assert rel_fro(got[(K, N)].numpy(), bt.grad.numpy()) <= 1e-2
    plan.close()


def test_grad_graph_norms(ctx):
    """rmsnorm(softmax(x @ w), gamma): gradients of x, w, gamma from the
    reference compiler's gradient graph (rmsnorm_grad, softmax_grad,
    reduce_sum, div, mul, transposed GEMMs)."""
    B, N = 64, 256
    rng = np.random.default_rng(13)
    x, w = half(rng, B, N, scale=0.3), half(rng, N, N, scale=0.3)
    gamma = (1 + 0.1 * rng.standard_normal(N)).astype(np.float16)
    s = O.softmax(f32(x) @ f32(w)).astype(np.float16)
    Y = O.rmsnorm(f32(s), f32(gamma), None, 1e-5).astype(np.float16)
    dY = half(rng, B, N)
    plan = bwpp.Plan(ctx, dump("norms", ".grad.dot"), None, dict(B=B, N=N))
    named = {plan.id(n) for n in ("x", "w", "gamma", "s")}
    unnamed = [v["id"] for v in plan.values() if v["input"] and v["id"] not in named]
    # the rmsnorm_grad node reads (s, gamma, dY): the seed is its third input;
    # the other unnamed input is the forward output Y
    steps = plan.describe()
    assert "rmsnorm_grad" in steps and len(unnamed) == 2
    keep = []
    dy_id, y_id = sorted(unnamed)  # dump order: v3 = dY seed, v6 = Y
    for key, arr in (("x", x), ("w", w), ("gamma", gamma), ("s", s), (dy_id, dY), (y_id, Y)):
        t = torch.from_numpy(np.ascontiguousarray(arr)).cuda()
        keep.append(t)
        plan.bind(key, t)
    plan.run()
    ctx.sync()
    got = {v["shape"]: plan.tensor(v["id"]).double().cpu().numpy() for v in plan.values() if v["output"]}
    xt, wt, gt = (torch.tensor(f32(u), dtype=torch.float64, requires_grad=True) for u in (x, w, gamma))
    st = torch.softmax(xt @ wt, -1)
    yt = st * torch.rsqrt((st * st).mean(-1, keepdim=True) + 1e-5) * gt
    yt.backward(torch.tensor(f32(dY), dtype=torch.float64))
    assert rel_fro(got[(N,)], gt.grad.numpy()) <= 2e-2
    assert rel_fro(got[(B, N)], xt.grad.numpy()) <= 3e-2
    assert rel_fro(got[(N, N)], wt.grad.numpy()) <= 3e-2
    plan.close()


def test_unbound_input_is_an_error(ctx):
    plan = bwpp.Plan(ctx, dump("matmul"), dump("matmul", ".mem.txt"), dict(M=8, K=16, N=32))
    with pytest.raises(bwpp.BwppError):
        plan.run()
    plan.close()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_graphs_in_other_storage_types(ctx, dtype):
    """The same reference dumps with every value declared f32 or bf16: the
    executor keeps that storage (f32 GEMM / attention operands are rounded to
    bf16 for the tensor cores, arithmetic stays fp32)."""
    tdt = {"f32": torch.float32, "bf16": torch.bfloat16}[dtype]
    tol = 2e-2 if dtype == "bf16" else 1e-2

    def run_dt(name, dims, inputs):
        dot = dump(name).replace(" f16 [", f" {dtype} [").replace("nf16 [", f"n{dtype} [")
        dot = dot.replace("\\nf16", f"\\n{dtype}").replace('"f16 ', f'"{dtype} ')
        mem = dump(name, ".mem.txt").replace(" f16 ", f" {dtype} ")
        plan = bwpp.Plan(ctx, dot, mem, dims)
        assert all(v["dtype"] == {"f32": "float32", "bf16": "bfloat16"}[dtype] for v in plan.values())
        for key, arr in inputs.items():
            plan.bind(key, torch.from_numpy(np.ascontiguousarray(arr, np.float32)).cuda().to(tdt))
        plan.run()
        ctx.sync()
        (out,) = [plan.tensor(v["id"]).float().cpu().numpy() for v in plan.values() if v["output"]]
        plan.close()
        return out

    rng = np.random.default_rng(21)
    M, K, N = 200, 256, 384
    a, b, bias = f32(half(rng, M, K, scale=0.5)), f32(half(rng, K, N, scale=0.5)), f32(half(rng, N, scale=0.1))
    out = run_dt("matmul_add_silu", dict(M=M, K=K, N=N), {"a": a, "b": b, "bias": bias})
    rb = lambda t: torch.from_numpy(t).to(torch.bfloat16).float().numpy()  # noqa: E731
    assert rel_fro(out, O.matmul(rb(a), rb(b), rb(bias) if dtype == "bf16" else bias, 1, 1)) <= tol
    B_, N_ = 64, 512
    x, w = f32(half(rng, B_, N_, scale=0.2)), f32(half(rng, N_, N_, scale=0.2))
    gamma = (1 + 0.1 * rng.standard_normal(N_)).astype(np.float32)
    out = run_dt("norms", dict(B=B_, N=N_), {"x": x, "w": w, "gamma": gamma})
    ref = O.rmsnorm(O.softmax(O.matmul(rb(x), rb(w))), gamma, None, 1e-5)
    assert rel_fro(out, ref) <= tol
    Bh, H, T, D = 1, 2, 256, 128
    q, k, v = (f32(half(rng, Bh, H, T, D, scale=0.3)) for _ in range(3))
    out = run_dt("attention", dict(B=Bh, H=H, T=T, D=D), {"q": q, "k": k, "v": v})
    assert rel_fro(out, O.attention_bhsd(rb(q), rb(k), rb(v), 1.0, 0)) <= tol


# ---- the swiglu and residual + norm patterns (spec/llm-primitives.md:17-22) --

def _silu(x):
    return x / (1 + np.exp(-x))


@pytest.mark.parametrize("fuse", [1, 0])
def test_swiglu_ffn_gate_in_the_gemm_epilogue(ctx, fuse):
    """silu(x W1) * (x W3) then W2: the gate multiplies in the W1 GEMM's
    epilogue (3 launches fused, 5 unfused)."""
    T, D, H = 200, 256, 384
    rng = np.random.default_rng(31)
    x = half(rng, T, D, scale=0.5)
    w1, w3 = half(rng, D, H, scale=0.1), half(rng, D, H, scale=0.1)
    w2 = half(rng, H, D, scale=0.1)
    outs, launches = run(ctx, "swiglu_ffn", dict(T=T, D=D, H=H), {"x": x, "w1": w1, "w3": w3, "w2": w2},
                         options=f"fuse={fuse}")
    g = O.matmul(f32(x), f32(w1))
    u = O.matmul(f32(x), f32(w3)).astype(np.float16)  # the graph stores u as f16
    a = (_silu(g) * f32(u)).astype(np.float16)
    ref = O.matmul(f32(a), f32(w2))
    (out,) = outs.values()
    assert rel_fro(out, ref) <= 3e-3
    assert launches == (3 if fuse else 5)


@pytest.mark.parametrize("fuse", [1, 0])
def test_swiglu_gate_standalone(ctx, fuse):
    """mul(silu(add(x, r)), y): the silu and mul run as one pass."""
    T, D = 300, 520
    rng = np.random.default_rng(32)
    x, r, y = half(rng, T, D), half(rng, T, D), half(rng, T, D)
    outs, launches = run(ctx, "swiglu_gate", dict(T=T, D=D), {"x": x, "r": r, "y": y},
                         options=f"fuse={fuse}")
    s = (f32(x) + f32(r)).astype(np.float16)
    ref = _silu(f32(s)) * f32(y)
    (out,) = outs.values()
    assert rel_fro(out, ref) <= 2e-3
    assert launches == (2 if fuse else 3)


@pytest.mark.parametrize("fuse", [1, 0])
@pytest.mark.parametrize("T,D", [(64, 256), (130, 1000)])
def test_residual_norm(ctx, fuse, T, D):
    """rmsnorm(add(x, r), g): one row kernel, the sum never stored."""
    rng = np.random.default_rng(33 + D)
    x, r = half(rng, T, D), half(rng, T, D)
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    outs, launches = run(ctx, "residual_norm", dict(T=T, D=D), {"x": x, "r": r, "g": g},
                         options=f"fuse={fuse}")
    h = (f32(x) + f32(r)).astype(np.float16)
    ref = O.rmsnorm(f32(h), f32(g), None, 1e-5)
    (out,) = outs.values()
    assert rel_fro(out, ref) <= 2e-3
    assert launches == (1 if fuse else 2)


@pytest.mark.parametrize("fuse", [1, 0])
@pytest.mark.parametrize("T,D", [(64, 256), (130, 1000)])
def test_residual_norm_in_f32_at_the_norm_tolerance(ctx, fuse, T, D):
    """The same graph with every value declared f32: no storage rounding is
    left, so the executor's residual + rmsnorm (fused, or add then norm)
    meets the north-star norm bound, 1e-5 relative, against the fp32 oracle."""
    rng = np.random.default_rng(35 + D)
    x, r = (rng.standard_normal((T, D)).astype(np.float32) for _ in range(2))
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    dot = dump("residual_norm").replace("\\nf16 [", "\\nf32 [").replace('"f16 [', '"f32 [')
    mem = dump("residual_norm", ".mem.txt").replace(" f16 ", " f32 ")
    plan = bwpp.Plan(ctx, dot, mem, dict(T=T, D=D), f"fuse={fuse}")
    assert all(v["dtype"] == "float32" for v in plan.values())
    for key, arr in {"x": x, "r": r, "g": g}.items():
        plan.bind(key, torch.from_numpy(arr).cuda())
    plan.run()
    ctx.sync()
    (out,) = [plan.tensor(v["id"]).cpu().numpy() for v in plan.values() if v["output"]]
    launches = plan.launches
    plan.close()
    ref = O.rmsnorm(x + r, g, None, 1e-5)
    assert rel_fro(out, ref) <= 1e-5
    assert launches == (1 if fuse else 2)


@pytest.mark.parametrize("fuse", [1, 0])
def test_attention_residual_norm_sum_stored(ctx, fuse):
    """h = x + attention(q, k, v); out = h + rmsnorm(h, g): the fused residual
    + norm stores h (read again by the last add), in the attention output's
    buffer as the memory plan has it."""
    T, D = 256, 128
    rng = np.random.default_rng(34)
    x, q, k, v = (half(rng, T, D, scale=0.3) for _ in range(4))
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    outs, launches = run(ctx, "attn_residual_norm", dict(T=T, D=D),
                         {"x": x, "q": q, "k": k, "v": v, "g": g}, options=f"fuse={fuse}")
    a = O.attention_bhsd(f32(q)[None, None], f32(k)[None, None], f32(v)[None, None], 1.0, 0)[0, 0]
    h = (f32(x) + a.astype(np.float16)).astype(np.float16)
    n = O.rmsnorm(f32(h), f32(g), None, 1e-5).astype(np.float16)
    ref = f32(h) + f32(n)
    (out,) = outs.values()
    assert rel_fro(out, ref) <= 1e-2
    assert launches == (3 if fuse else 7)


# ---- launch plans written by `bwppc --target cuda` ------------------------------

def _launch_fixtures():
    out = []
    for f in sorted(os.listdir(PLANS)):
        if f.endswith(".plan") and "V32000" not in f:  # the bench-size plan runs in bench.py
            name, tag = f[:-5].split("@")
            dims = {}
            for part in tag.split("_"):
                i = next(j for j, ch in enumerate(part) if ch.isdigit())
                dims[part[:i]] = int(part[i:])
            out.append((name, dims, f))
    return out


@pytest.mark.parametrize("name,dims,fname", _launch_fixtures())
def test_compiler_launch_plan_runs_like_the_dump(ctx, name, dims, fname):
    """The compiler's launch plan and the executor's lowering of the graph
    dumps are the same program: on the same inputs every output is bit for
    bit the same, with the same launches (their numerics against the oracle
    are checked at these dims by the tests above)."""
    if name == "permute_max.grad":
        pytest.skip("the dump cannot carry the permute's axes (its own test below)")
    with open(os.path.join(PLANS, fname)) as f:
        launch = bwpp.Plan(ctx, f.read())
    if name.endswith(".grad"):  # gradient graph: no memory-plan dump for it
        lowered = bwpp.Plan(ctx, dump(name[:-5], ".grad.dot"), None, dims)
    else:
        lowered = bwpp.Plan(ctx, dump(name), dump(name, ".mem.txt"), dims)
    rng = np.random.default_rng(len(fname))
    keep = []
    for v in lowered.values():
        if not v["input"]:
            continue
        shape = v["shape"]
        scale = 1.0 if len(shape) == 1 else shape[-1] ** -0.5
        arr = half(rng, *shape, scale=scale)
        if len(shape) == 1:
            arr = (1 + 0.1 * arr).astype(np.float16)
        t = torch.from_numpy(arr).cuda()
        keep.append(t)
        lowered.bind(v["id"], t)
        launch.bind(v["id"], t)
    lowered.run()
    launch.run()
    ctx.sync()
    outs = [v["id"] for v in lowered.values() if v["output"]]
    assert outs
    for vid in outs:
        a = launch.tensor(vid).cpu()
        b = lowered.tensor(vid).cpu()
        assert torch.equal(a, b), (fname, vid)
        assert bool(torch.isfinite(a.float()).all())
    assert launch.launches == lowered.launches
    launch.close()
    lowered.close()


def test_tiny_model_forward_from_the_compiler_launch_plan(ctx):
    """examples/tiny_model.bwpp compiled with --target cuda, against the fp32
    oracle composition."""
    T, D, H, V = 256, 128, 256, 512
    rng = np.random.default_rng(7)
    p = {"x": half(rng, T, D)}
    for pre in ("1", "2"):
        for w in ("wq", "wk", "wv", "wo"):
            p[w + pre] = half(rng, D, D, scale=D ** -0.5)
        p["w1" + pre] = half(rng, D, H, scale=D ** -0.5)
        p["w2" + pre] = half(rng, H, D, scale=H ** -0.5)
        p["g1" + pre] = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
        p["g2" + pre] = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    p["wcls"] = half(rng, D, V, scale=D ** -0.5)
    with open(os.path.join(PLANS, "tiny_model@T256_D128_H256_V512.plan")) as f:
        plan = bwpp.Plan(ctx, f.read())
    keep = []
    for key, arr in p.items():
        t = torch.from_numpy(arr).cuda()
        keep.append(t)
        plan.bind(key, t)
    plan.run()
    ctx.sync()
    (out,) = [plan.tensor(v["id"]).float().cpu().numpy() for v in plan.values() if v["output"]]
    assert out.shape == (T, V)
    assert rel_fro(out, tiny_forward_ref({k: f32(v) for k, v in p.items()})) <= 3e-2
    assert plan.launches == 20
    plan.close()


# ---- permute and reduce_max (compiler/graph_ir.c:496-548, 663-695, 1672-1690, 1798-1821) --

def _plan_from(ctx, fname, inputs):
    with open(os.path.join(PLANS, fname)) as f:
        plan = bwpp.Plan(ctx, f.read())
    keep = []
    ids = [v["id"] for v in plan.values() if v["input"]]
    for vid, arr in zip(ids, inputs):
        t = torch.from_numpy(np.ascontiguousarray(arr)).cuda()
        keep.append(t)
        plan.bind(vid, t)
    plan.run()
    ctx.sync()
    outs = [plan.tensor(v["id"]).float().cpu().numpy() for v in plan.values() if v["output"]]
    plan.close()
    return outs


def test_permute_and_reduce_max_forward(ctx):
    """permute(x, [0,2,1,3]) then reduce_max over the last axis (f16), exact."""
    B, T, H, D = 2, 128, 4, 64
    x = half(np.random.default_rng(41), B, T, H, D)
    (out,) = _plan_from(ctx, "permute_max@B2_T128_H4_D64.plan", [x])
    ref = np.transpose(f32(x), (0, 2, 1, 3)).max(axis=3, keepdims=True)
    assert out.shape == (B, H, T, 1) and np.array_equal(out, ref)
    lowered = bwpp.Plan(ctx, dump("permute_max"), dump("permute_max", ".mem.txt"), dict(B=B, T=T, H=H, D=D))
    lowered.bind("x", torch.from_numpy(x).cuda())
    lowered.run()
    ctx.sync()
    (vid,) = [v["id"] for v in lowered.values() if v["output"]]
    assert np.array_equal(lowered.tensor(vid).float().cpu().numpy(), ref)
    lowered.close()


def test_permute_and_reduce_max_gradient(ctx):
    """The gradient graph (mask of every tied maximum, dy broadcast, their
    product, the inverse permute) against the reference's mask / grad
    semantics (oracle restatement of runtime/cpu/bwpp_cpu_ref.c:146-219)."""
    B, T, H, D = 2, 128, 4, 64
    rng = np.random.default_rng(42)
    x = half(rng, B, T, H, D)
    y = np.ascontiguousarray(np.transpose(x, (0, 2, 1, 3)))          # forward activation
    dy = half(rng, B, H, T, 1)
    # inputs in value order: x, the seed dY [B,H,T,1], the activation y
    (dx,) = _plan_from(ctx, "permute_max.grad@B2_T128_H4_D64.plan", [x, dy, y])
    rows = f32(y).reshape(-1, D)
    mask = O.reduce_max_mask(rows, 1)
    g = O.reduce_max_grad(mask, f32(dy).reshape(-1), 1).reshape(B, H, T, D)
    ref = np.transpose(g.astype(np.float16), (0, 2, 1, 3)).astype(np.float32)
    assert dx.shape == (B, T, H, D) and np.array_equal(dx, ref)


def test_row_max_gradient_with_ties(ctx):
    """f32 rows with many ties: every tied maximum takes the gradient, bit for
    bit as the reference's reduce_max mask / grad pair."""
    R, C = 300, 1000
    rng = np.random.default_rng(43)
    x = rng.integers(0, 5, (R, C)).astype(np.float32)  # ties everywhere
    dy = rng.standard_normal((R, 1)).astype(np.float32)
    (mx,) = _plan_from(ctx, "row_max@R300_C1000.plan", [x])
    assert np.array_equal(mx, x.max(axis=1, keepdims=True))
    (dx,) = _plan_from(ctx, "row_max.grad@R300_C1000.plan", [x, dy])
    mask = O.reduce_max_mask(x, 1)
    assert np.array_equal(dx, O.reduce_max_grad(mask, dy.reshape(-1), 1))
