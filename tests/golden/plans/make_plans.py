#!/usr/bin/env python3
"""Regenerates the graph / memory-plan dumps in this folder with the
reference compiler itself.

The reference compiler is built unmodified from its sources by
`make -C oracle bwppc` (into oracle/_ref/bwppc, git-ignored) and run on the
reference's own examples and on the test sources in src/ (written for this
repository in the reference DSL: the swiglu and residual + norm patterns,
permute and reduce_max):
    bwppc <example>.bwpp <tmp>.metal --entry <fn> --dot <name>.dot
          --grad-dot <name>.grad.dot --mem-plan <name>.mem.txt
It also builds `bwppc` with this package's CUDA target
(`make -C bluewolf-plus-plus_b200/compiler`, the reference sources with
main.c patched) and writes launch plans, <name>@<dims>.plan, for the dims the
executor tests use:
    bwppc <example>.bwpp <name>@<dims>.plan --entry <fn> --target cuda --dims ...
and, for gradient graphs, <name>.grad@<dims>.plan with --grad-plan.
The dumps and plans are committed so the executor tests run where the
reference tree is absent (the GPU box).  Run from anywhere: python tests/golden/plans/make_plans.py
The reference checkout is taken from $BWPP_REFERENCE, else from a directory
named `reference` beside this repository.
"""
import os
import subprocess
import sys
import tempfile

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(os.path.dirname(HERE)))
REF = os.environ.get("BWPP_REFERENCE", os.path.join(os.path.dirname(ROOT), "reference"))
BWPPC = os.path.join(ROOT, "oracle", "_ref", "bwppc")

# (dump name, example file, entry function)
CASES = [
    ("matmul", "matmul", "matmul"),
    ("matmul_add_silu", "matmul_add_silu", "fused"),
    ("matmul_add_bias_reshape", "matmul_add_bias_reshape", "fused"),
    ("multi_fn_bias", "multi_fn_bias", "block_b"),
    ("norms", "norms", "norms"),
    ("attention", "attention", "attention"),
    ("tiny_attn", "tiny_model", "attn"),
    ("tiny_ffn", "tiny_model", "ffn"),
    ("tiny_block", "tiny_model", "block"),
    ("tiny_model", "tiny_model", "tiny_model"),
    ("swiglu_ffn", "src/swiglu_ffn", "swiglu_ffn"),
    ("swiglu_gate", "src/swiglu_ffn", "gate"),
    ("attn_residual_norm", "src/residual_norm", "attn_residual_norm"),
    ("residual_norm", "src/residual_norm", "residual_norm"),
    ("permute_max", "src/permute_max", "permute_max"),
    ("row_max", "src/permute_max", "row_max"),
]


# launch plans: (dump name, dims) -- the dims of the executor's GPU tests
LAUNCH = [
    ("matmul_add_silu", dict(M=200, K=256, N=384)),
    ("matmul_add_bias_reshape", dict(M=129, K=136, N=264)),
    ("norms", dict(B=96, N=512)),
    ("attention", dict(B=2, H=3, T=256, D=64)),
    ("attention", dict(B=2, H=3, T=256, D=128)),
    ("attention", dict(B=2, H=3, T=256, D=96)),
    ("tiny_block", dict(T=128, D=256, H=512)),
    ("tiny_model", dict(T=256, D=128, H=256, V=512)),
    ("tiny_model", dict(T=128, D=256, H=512, V=1000)),
    ("tiny_model", dict(T=8192, D=1024, H=4096, V=32000)),
    ("swiglu_ffn", dict(T=200, D=256, H=384)),
    ("swiglu_gate", dict(T=300, D=520)),
    ("residual_norm", dict(T=64, D=256)),
    ("residual_norm", dict(T=130, D=1000)),
    ("attn_residual_norm", dict(T=256, D=128)),
    ("permute_max", dict(B=2, T=128, H=4, D=64)),
    ("row_max", dict(R=300, C=1000)),
]
# gradient graphs (--grad-plan): <name>.grad@<dims>.plan
GRAD_LAUNCH = [
    ("matmul_add_silu", dict(M=192, K=128, N=256)),
    ("norms", dict(B=64, N=256)),
    ("permute_max", dict(B=2, T=128, H=4, D=64)),
    ("row_max", dict(R=300, C=1000)),
]
CUDA_BWPPC = os.path.join(ROOT, "bluewolf-plus-plus_b200", "compiler", "_build", "bwppc")


def tag(dims):
    return "_".join(f"{k}{v}" for k, v in dims.items())


def main():
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "bwppc", f"REF={REF}"], check=True)
    subprocess.run(["make", "-C", os.path.join(ROOT, "bluewolf-plus-plus_b200", "compiler"),
                    f"REF={REF}"], check=True)
    if not os.path.exists(BWPPC):
        sys.exit("oracle/_ref/bwppc was not built (reference tree missing?)")
    with tempfile.TemporaryDirectory() as tmp:
        for name, example, entry in CASES:
            src = (os.path.join(HERE, example + ".bwpp") if example.startswith("src/")
                   else os.path.join(REF, "examples", example + ".bwpp"))
            out = lambda ext: os.path.join(HERE, name + ext)
            subprocess.run([BWPPC, src, os.path.join(tmp, name + ".metal"), "--entry", entry,
                            "--dot", out(".dot"), "--grad-dot", out(".grad.dot"),
                            "--mem-plan", out(".mem.txt")], check=True)
            print("wrote", name)
    srcs = {name: (example, entry) for name, example, entry in CASES}
    for name, dims in LAUNCH:
        example, entry = srcs[name]
        src = (os.path.join(HERE, example + ".bwpp") if example.startswith("src/")
               else os.path.join(REF, "examples", example + ".bwpp"))
        out = os.path.join(HERE, f"{name}@{tag(dims)}.plan")
        subprocess.run([CUDA_BWPPC, src, out, "--entry", entry, "--target", "cuda", "--dims",
                        ",".join(f"{k}={v}" for k, v in dims.items())], check=True)
        print("wrote", os.path.basename(out))
    with tempfile.TemporaryDirectory() as tmp:
        for name, dims in GRAD_LAUNCH:
            example, entry = srcs[name]
            src = (os.path.join(HERE, example + ".bwpp") if example.startswith("src/")
                   else os.path.join(REF, "examples", example + ".bwpp"))
            out = os.path.join(HERE, f"{name}.grad@{tag(dims)}.plan")
            subprocess.run([CUDA_BWPPC, src, os.path.join(tmp, "fwd.plan"), "--entry", entry,
                            "--target", "cuda", "--dims", ",".join(f"{k}={v}" for k, v in dims.items()),
                            "--grad-plan", out], check=True)
            print("wrote", os.path.basename(out))


if __name__ == "__main__":
    main()
