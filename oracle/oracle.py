"""numpy front-end of the CPU checkers.  TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs import this module; the CUDA runtime never does.

  Oracle   -- this repo's C restatement (oracle/bwpp_oracle.c, libbwpp_oracle.so)
  Ref      -- the reference's own runtime/cpu/bwpp_cpu_ref.c compiled from the
              reference sources into oracle/_ref/libbwpp_cpu_ref.so (None when
              that file is absent)

Parity pin: tests/test_oracle.py checks Oracle against Ref bit-for-bit and
against the golden fixtures under tests/golden/ (made by running Ref).
The extensions (layernorm, norm backward, argmax, batched attention) have no
reference counterpart ("parity unpinned by the reference") and are checked
against float64 numpy there.

Inputs: the generators below are the seeded synthetic stand-ins for the
benchmark configs (the reference ships no datasets).
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_LIB = os.path.join(HERE, "libbwpp_oracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libbwpp_cpu_ref.so")

_f = C.POINTER(C.c_float)
_u16 = C.POINTER(C.c_uint16)
_u32p = C.POINTER(C.c_uint32)
_u32, _i32, _f32, _sz = C.c_uint32, C.c_int, C.c_float, C.c_size_t

_REF_SIGS = {
    "matmul_f32": [_f, _f, _f, _u32, _u32, _u32, _u32, _u32, _u32, _f, _i32, _i32],
    "softmax_f32": [_f, _f, _u32, _u32, _u32],
    "rmsnorm_f32": [_f, _f, _f, _f, _u32, _u32, _u32, _f32],
    "attention_f32": [_f, _f, _f, _f] + [_u32] * 8,
    "reduce_max_mask_f32": [_f, _f, _u32, _u32, _i32],
    "reduce_max_grad_f32": [_f, _f, _f, _u32, _u32, _i32],
}
_EXT_SIGS = {
    "reduce_max_argmax_f32": [_f, _f, _u32p, _u32, _u32, _u32],
    "reduce_max_bwd_f32": [_u32p, _f, _f, _u32, _u32, _u32],
    "layernorm_f32": [_f, _f, _f, _f, _u32, _u32, _u32, _f32],
    "rmsnorm_bwd_f32": [_f, _f, _f, _f, _f, _f, _u32, _u32, _u32, _f32],
    "layernorm_bwd_f32": [_f, _f, _f, _f, _f, _f, _u32, _u32, _u32, _f32],
    "attention_bhsd_f32": [_f, _f, _f, _f, _u32, _u32, _u32, _u32, _u32, _f32, _i32, _u32, _u32],
    "attention_bhsd_fast_f32": [_f, _f, _f, _f, _u32, _u32, _u32, _u32, _u32, _f32, _i32, _u32, _u32],
    "f32_to_bf16": [_f, _u16, _sz],
    "bf16_to_f32": [_u16, _f, _sz],
    "silu_grad_f32": [_f, _f, _f, _sz],
    "softmax_grad_f32": [_f, _f, _f, _u32, _u32, _u32],
    "reduce_sum_f32": [_f, _f, _u32, _u32, _u32, _i32],
    "broadcast_f32": [_f, _f, _u32, _u32, _u32, _i32],
}


def _fp(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous, (a.dtype, a.flags)
    return a.ctypes.data_as(_f)


def _u32ptr(a):
    assert a.dtype == np.uint32 and a.flags.c_contiguous
    return a.ctypes.data_as(_u32p)


class _Lib:
    def __init__(self, path, prefix, sigs):
        self.path = path
        self.lib = C.CDLL(path)
        for name, args in sigs.items():
            fn = getattr(self.lib, prefix + name)
            fn.argtypes = args
            fn.restype = None
            setattr(self, name, fn)


_oracle = None
_ref = None


def oracle_lib() -> _Lib:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_LIB):
            raise ImportError(f"{ORACLE_LIB} missing: run `make -C oracle`")
        _oracle = _Lib(ORACLE_LIB, "bwpp_oracle_", {**_REF_SIGS, **_EXT_SIGS})
    return _oracle


def ref_lib():
    """The reference's own CPU library, or None when it was not built here."""
    global _ref
    if _ref is None and os.path.exists(REF_LIB):
        _ref = _Lib(REF_LIB, "bwpp_cpu_", _REF_SIGS)
    return _ref


# ---------------------------------------------------------------------------
# numpy wrappers (same argument meaning as runtime/cpu/bwpp_cpu_ref.h)
# ---------------------------------------------------------------------------

def matmul(a, b, bias=None, silu=False, add=False, lib=None):
    lib = lib or oracle_lib()
    M, K = a.shape
    N = b.shape[1]
    c = np.zeros((M, N), np.float32)
    lib.matmul_f32(_fp(a), _fp(b), _fp(c), M, N, K, K, N, N, _fp(bias), int(silu), int(add))
    return c


def softmax(x, lib=None):
    lib = lib or oracle_lib()
    y = np.zeros_like(x)
    lib.softmax_f32(_fp(x), _fp(y), x.shape[0], x.shape[1], x.shape[1])
    return y


def rmsnorm(x, gamma=None, beta=None, eps=1e-5, lib=None):
    lib = lib or oracle_lib()
    y = np.zeros_like(x)
    lib.rmsnorm_f32(_fp(x), _fp(y), _fp(gamma), _fp(beta), x.shape[0], x.shape[1], x.shape[1], eps)
    return y


def attention2d(q, k, v, lib=None):
    """runtime/cpu/bwpp_cpu_ref.c:92-144 on dense 2-D q [M,K], k [N,K], v [N,D]."""
    lib = lib or oracle_lib()
    M, K = q.shape
    N, D = v.shape
    o = np.zeros((M, D), np.float32)
    lib.attention_f32(_fp(q), _fp(k), _fp(v), _fp(o), M, N, K, D, K, K, D, D)
    return o


def reduce_max_mask(x, axis=1, lib=None):
    lib = lib or oracle_lib()
    m = np.zeros_like(x)
    lib.reduce_max_mask_f32(_fp(x), _fp(m), x.shape[0], x.shape[1], axis)
    return m


def reduce_max_grad(mask, dy, axis=1, lib=None):
    lib = lib or oracle_lib()
    dx = np.zeros_like(mask)
    lib.reduce_max_grad_f32(_fp(mask), _fp(dy), _fp(dx), mask.shape[0], mask.shape[1], axis)
    return dx


def reduce_max_argmax(x):
    rows, cols = x.shape
    mx = np.zeros(rows, np.float32)
    am = np.zeros(rows, np.uint32)
    oracle_lib().reduce_max_argmax_f32(_fp(x), _fp(mx), _u32ptr(am), rows, cols, cols)
    return mx, am


def reduce_max_bwd(argmax, dy, cols):
    rows = argmax.shape[0]
    dx = np.zeros((rows, cols), np.float32)
    oracle_lib().reduce_max_bwd_f32(_u32ptr(argmax), _fp(dy), _fp(dx), rows, cols, cols)
    return dx


def layernorm(x, gamma=None, beta=None, eps=1e-5):
    y = np.zeros_like(x)
    oracle_lib().layernorm_f32(_fp(x), _fp(y), _fp(gamma), _fp(beta), x.shape[0], x.shape[1],
                               x.shape[1], eps)
    return y


def norm_bwd(x, gamma, dy, eps=1e-5, centered=False):
    rows, cols = x.shape
    dx = np.zeros_like(x)
    dg = np.zeros(cols, np.float32)
    db = np.zeros(cols, np.float32)
    fn = oracle_lib().layernorm_bwd_f32 if centered else oracle_lib().rmsnorm_bwd_f32
    fn(_fp(x), _fp(gamma), _fp(dy), _fp(dx), _fp(dg), _fp(db), rows, cols, cols, eps)
    return dx, dg, db


def attention_bhsd(q, k, v, scale, causal, rows=None, fast=True):
    """Batched [B,H,S,D] attention; rows=(begin, end) restricts the query rows."""
    B, H, Sq, D = q.shape
    Skv = k.shape[2]
    o = np.zeros((B, H, Sq, D), np.float32)
    r0, r1 = rows if rows is not None else (0, Sq)
    fn = oracle_lib().attention_bhsd_fast_f32 if fast else oracle_lib().attention_bhsd_f32
    fn(_fp(q), _fp(k), _fp(v), _fp(o), B, H, Sq, Skv, D, scale, int(causal), r0, r1)
    return o


def silu_grad(x, dy):
    x, dy = (np.ascontiguousarray(t, np.float32) for t in (x, dy))
    dx = np.zeros_like(x)
    oracle_lib().silu_grad_f32(_fp(x), _fp(dy), _fp(dx), x.size)
    return dx


def softmax_grad(y, dy):
    rows, cols = y.shape
    dx = np.zeros_like(y)
    oracle_lib().softmax_grad_f32(_fp(y), _fp(dy), _fp(dx), rows, cols, cols)
    return dx


def reduce_sum(x, axis):
    rows, cols = x.shape
    out = np.zeros(rows if axis == 1 else cols, np.float32)
    oracle_lib().reduce_sum_f32(_fp(x), _fp(out), rows, cols, cols, int(axis))
    return out


def broadcast(src, rows, cols, axis):
    dst = np.zeros((rows, cols), np.float32)
    oracle_lib().broadcast_f32(_fp(np.ascontiguousarray(src, np.float32)), _fp(dst), rows, cols,
                               cols, int(axis))
    return dst


def f32_to_bf16(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    oracle_lib().f32_to_bf16(_fp(x), out.ctypes.data_as(_u16), x.size)
    return out


def bf16_to_f32(h):
    h = np.ascontiguousarray(h, np.uint16)
    out = np.empty(h.shape, np.float32)
    oracle_lib().bf16_to_f32(h.ctypes.data_as(_u16), _fp(out), h.size)
    return out


def round_bf16(x):
    """fp32 values rounded to bf16 (nearest even) and back: the exact values a bf16 kernel sees."""
    return bf16_to_f32(f32_to_bf16(x))


# ---------------------------------------------------------------------------
# threaded row-split runner for CPU-baseline timing (ctypes drops the GIL)
# ---------------------------------------------------------------------------

def run_rows_threaded(fn, rows: int, threads: int):
    """Calls fn(r0, r1) on `threads` disjoint row ranges concurrently."""
    threads = max(1, min(threads, rows))
    step = (rows + threads - 1) // threads
    ts = [threading.Thread(target=fn, args=(i * step, min(rows, (i + 1) * step)))
          for i in range(threads) if i * step < rows]
    for t in ts:
        t.start()
    for t in ts:
        t.join()


def ref_matmul_rows(lib, a, b, c, bias, silu, add, r0, r1):
    """lib.matmul_f32 on rows [r0, r1) of the dense problem (M=r1-r0 view)."""
    M, K = a.shape
    N = b.shape[1]
    if r1 <= r0:
        return
    pa = C.cast(C.c_void_p(a.ctypes.data + r0 * K * 4), _f)
    pc = C.cast(C.c_void_p(c.ctypes.data + r0 * N * 4), _f)
    lib.matmul_f32(pa, _fp(b), pc, r1 - r0, N, K, K, N, N, _fp(bias), int(silu), int(add))


def cpu_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1
