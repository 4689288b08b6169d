"""Regenerates tests/golden/ref_golden.npz by running the REFERENCE's own CPU
library (runtime/cpu/bwpp_cpu_ref.c compiled from the reference sources into
oracle/_ref/libbwpp_cpu_ref.so by `make -C oracle ref`).

Cases:
  * the known-answer setups of the reference's tests, with their ramp fill
    (i*cols + j + 1) * scale (runtime/cpu/test_metal_parity.c:36-42):
      matmul 4x4x4, a*0.1, b*0.05, bias 0.01*(i+1), every epilogue
        (test_metal_parity.c:86-131); softmax / rmsnorm 2x4 x*0.1 (136-231);
      attention M=2 N=3 K=4 D=5, q*0.03 k*0.04 v*0.02 (233-302);
      reduce_max 2x3 iota, dy = r+1 (test_reduce_max.c:5-55);
      bench matmul 256^3, a*0.01 b*0.02 (bench/bench_cpu.c:82-83)
  * seeded random cases with awkward sizes, ties, negative values.

Usage: python tests/golden/make_golden.py   (needs oracle/_ref built here)
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as O  # noqa: E402


def ramp(rows, cols, scale):
    i = np.arange(rows * cols, dtype=np.float64).reshape(rows, cols)
    return ((i + 1).astype(np.float32) * np.float32(scale)).astype(np.float32)


def main():
    ref = O.ref_lib()
    if ref is None:
        raise SystemExit("oracle/_ref/libbwpp_cpu_ref.so missing: run `make -C oracle ref`")
    g = {}
    # --- reference test setups --------------------------------------------
    a, b = ramp(4, 4, 0.1), ramp(4, 4, 0.05)
    bias = (0.01 * np.arange(1, 5)).astype(np.float32)
    g["mm4_a"], g["mm4_b"], g["mm4_bias"] = a, b, bias
    for add in (0, 1):
        for silu in (0, 1):
            g[f"mm4_out_add{add}_silu{silu}"] = O.matmul(a, b, bias, silu, add, lib=ref)
    x = ramp(2, 4, 0.1)
    g["sm_x"] = x
    g["sm_out"] = O.softmax(x, lib=ref)
    g["rms_x"] = x
    g["rms_gamma"] = np.ones(4, np.float32)
    g["rms_out"] = O.rmsnorm(x, g["rms_gamma"], None, 1e-5, lib=ref)
    q, k, v = ramp(2, 4, 0.03), ramp(3, 4, 0.04), ramp(3, 5, 0.02)
    g["att_q"], g["att_k"], g["att_v"] = q, k, v
    g["att_out"] = O.attention2d(q, k, v, lib=ref)
    xi = np.arange(6, dtype=np.float32).reshape(2, 3)
    dy_r = np.array([1, 2], np.float32)
    g["rmax_x"], g["rmax_dy"] = xi, dy_r
    g["rmax_mask1"] = O.reduce_max_mask(xi, 1, lib=ref)
    g["rmax_grad1"] = O.reduce_max_grad(g["rmax_mask1"], dy_r, 1, lib=ref)
    g["rmax_mask0"] = O.reduce_max_mask(xi, 0, lib=ref)
    g["rmax_grad0"] = O.reduce_max_grad(g["rmax_mask0"], np.array([1, 2, 3], np.float32), 0, lib=ref)
    a, b = ramp(256, 256, 0.01), ramp(256, 256, 0.02)
    g["bench_mm_out"] = O.matmul(a, b, np.zeros(256, np.float32), 0, 0, lib=ref)

    # --- seeded random cases --------------------------------------------------
    rng = np.random.default_rng(20261201)
    a = rng.standard_normal((17, 29)).astype(np.float32)
    b = rng.standard_normal((29, 33)).astype(np.float32)
    bias = rng.uniform(-0.1, 0.1, 33).astype(np.float32)
    g["rmm_a"], g["rmm_b"], g["rmm_bias"] = a, b, bias
    g["rmm_out"] = O.matmul(a, b, bias, 1, 1, lib=ref)
    x = rng.standard_normal((5, 37)).astype(np.float32)
    gam = (1 + 0.1 * rng.standard_normal(37)).astype(np.float32)
    bet = (0.1 * rng.standard_normal(37)).astype(np.float32)
    g["rrms_x"], g["rrms_gamma"], g["rrms_beta"] = x, gam, bet
    g["rrms_out"] = O.rmsnorm(x, gam, bet, 1e-5, lib=ref)
    x = (3 * rng.standard_normal((3, 50))).astype(np.float32)
    g["rsm_x"] = x
    g["rsm_out"] = O.softmax(x, lib=ref)
    q = rng.standard_normal((7, 16)).astype(np.float32)
    k = rng.standard_normal((9, 16)).astype(np.float32)
    v = rng.standard_normal((9, 12)).astype(np.float32)
    g["ratt_q"], g["ratt_k"], g["ratt_v"] = q, k, v
    g["ratt_out"] = O.attention2d(q, k, v, lib=ref)
    x = rng.integers(-3, 3, (6, 10)).astype(np.float32)  # many ties
    dyr = rng.standard_normal(6).astype(np.float32)
    dyc = rng.standard_normal(10).astype(np.float32)
    g["rrmax_x"], g["rrmax_dyr"], g["rrmax_dyc"] = x, dyr, dyc
    for axis, dy in ((0, dyc), (1, dyr)):
        m = O.reduce_max_mask(x, axis, lib=ref)
        g[f"rrmax_mask{axis}"] = m
        g[f"rrmax_grad{axis}"] = O.reduce_max_grad(m, dy, axis, lib=ref)

    out = os.path.join(HERE, "ref_golden.npz")
    np.savez_compressed(out, **g)
    print(f"wrote {out}: {len(g)} arrays")


if __name__ == "__main__":
    main()
