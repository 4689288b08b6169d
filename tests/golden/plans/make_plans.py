#!/usr/bin/env python3
"""Regenerates the graph / memory-plan dumps in this folder with the
reference compiler itself.

The reference compiler is built unmodified from its sources by
`make -C oracle bwppc` (into oracle/_ref/bwppc, git-ignored) and run on the
reference's own examples and on the test sources in src/ (written for this
repository in the reference DSL: the swiglu and residual + norm patterns):
    bwppc <example>.bwpp <tmp>.metal --entry <fn> --dot <name>.dot
          --grad-dot <name>.grad.dot --mem-plan <name>.mem.txt
The dumps are committed so the executor tests run where the reference tree
is absent (the GPU box).  Run from anywhere: python tests/golden/plans/make_plans.py
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
]


def main():
    subprocess.run(["make", "-C", os.path.join(ROOT, "oracle"), "bwppc", f"REF={REF}"], check=True)
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


if __name__ == "__main__":
    main()
