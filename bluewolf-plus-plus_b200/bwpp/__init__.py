"""Python view of the BW++ B200 runtime (lib/libbwpp_cuda.so) through its C ABI.

This module is a thin ctypes layer over include/bwpp_cuda.h, used by the test
suite, bench.py and __graft_entry__.  It adds no compute of its own: every op
below is one call into the CUDA library, and importing it fails loudly when the
library has not been built (there is no CPU fallback).

Argument order and meaning follow the reference's runtime/cpu/bwpp_cpu_ref.h
and runtime/metal/dispatch_stub.h (see the C header for citations).
"""
from __future__ import annotations

import ctypes as C
import os
import re

_HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(_HERE)
REPO_ROOT = os.path.dirname(PKG_ROOT)
LIB_PATH = os.path.join(PKG_ROOT, "lib", "libbwpp_cuda.so")
HEADER_PATH = os.path.join(REPO_ROOT, "include", "bwpp_cuda.h")

OK = 0
ERR = 1
ERR_ARG = 2
ERR_CUDA = 3
ERR_TIMEOUT = 4
ERR_NOMEM = 5
ERR_UNSUPPORTED = 6

_u32, _u64, _i32, _f32, _vp, _sz = C.c_uint32, C.c_uint64, C.c_int, C.c_float, C.c_void_p, C.c_size_t
_cp = C.c_char_p


class BwppError(RuntimeError):
    def __init__(self, status, message=""):
        super().__init__(f"bwpp status {status}: {message}")
        self.status = status


class MatmulParams(C.Structure):
    _fields_ = [(n, _u32) for n in ("M", "N", "K", "lda", "ldb", "ldc")]


class SoftmaxParams(C.Structure):
    _fields_ = [(n, _u32) for n in ("rows", "cols", "ld")]


class RmsnormParams(C.Structure):
    _fields_ = [("rows", _u32), ("cols", _u32), ("ld", _u32), ("eps", _f32)]


class AttentionParams(C.Structure):
    _fields_ = [(n, _u32) for n in ("M", "N", "K", "D", "ldq", "ldk", "ldv", "ldo")]


class GemmParams(C.Structure):
    _fields_ = [(n, _u32) for n in ("M", "N", "K", "lda", "ldb", "ldc", "ldr")] + \
               [(n, _i32) for n in ("a_mn_major", "b_mn_major", "out_bf16", "apply_silu")] + \
               [("bias", _vp), ("residual", _vp)]


class TinyModelConfig(C.Structure):
    _fields_ = [(n, _u32) for n in ("layers", "d_model", "heads", "head_dim", "ffn", "batch", "seq")] + \
               [("eps", _f32)]


class Arena(C.Structure):
    _fields_ = [("buffer", _vp), ("capacity", _sz), ("offset", _sz)]


# name -> (restype, argtypes)
_SIGS = {
    "bwpp_cuda_arena_init": (_i32, [C.POINTER(Arena), _sz, _i32]),
    "bwpp_cuda_arena_alloc": (_vp, [C.POINTER(Arena), _sz, _sz]),
    "bwpp_cuda_arena_reset": (None, [C.POINTER(Arena)]),
    "bwpp_cuda_arena_destroy": (None, [C.POINTER(Arena)]),
    "bwpp_cuda_ctx_create": (_i32, [C.POINTER(_vp), _i32, _vp]),
    "bwpp_cuda_ctx_destroy": (_i32, [_vp]),
    "bwpp_cuda_ctx_set_stream": (_i32, [_vp, _vp]),
    "bwpp_cuda_ctx_set_workspace": (_i32, [_vp, _vp, _sz]),
    "bwpp_cuda_norm_bwd_workspace_size": (_sz, [_vp, _u32, _u32]),
    "bwpp_cuda_sync": (_i32, [_vp]),
    "bwpp_cuda_copy": (_i32, [_vp, _vp, _vp, _sz]),
    "bwpp_cuda_status_string": (_cp, [_i32]),
    "bwpp_cuda_ctx_last_error": (_cp, [_vp]),
    "bwpp_cuda_device_count": (_i32, []),
    "bwpp_cuda_selftest_wait_timeout": (_i32, [_vp, _u32]),
    "bwpp_cuda_selftest_occupy": (_i32, [_vp, _vp, _u32, _u32, _u32]),
    "bwpp_cuda_matmul_bf16": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _vp, _i32, _i32]),
    "bwpp_cuda_gemm_bf16_ex": (_i32, [_vp, _vp, _vp, _vp, C.POINTER(GemmParams)]),
    "bwpp_cuda_attention_bf16": (_i32, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _f32, _i32]),
    "bwpp_cuda_rmsnorm_fwd_f32": (_i32, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _f32]),
    "bwpp_cuda_rmsnorm_bwd_f32": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _f32]),
    "bwpp_cuda_rmsnorm_bwd_f32_noalloc": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _f32, _vp]),
    "bwpp_cuda_layernorm_fwd_f32": (_i32, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _f32]),
    "bwpp_cuda_layernorm_bwd_f32": (_i32, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _f32]),
    "bwpp_cuda_reduce_max_fwd_f32": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32]),
    "bwpp_cuda_reduce_max_bwd_f32": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32]),
    "bwpp_cuda_reduce_max_mask_ex": (_i32, [_vp, _vp, _vp, _u32, _u32, _i32]),
    "bwpp_cuda_reduce_max_grad_ex": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _i32]),
    "bwpp_cuda_softmax_fwd_f32": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32]),
    "bwpp_cuda_silu_grad_f32": (_i32, [_vp, _vp, _vp, _vp, C.c_size_t]),
    "bwpp_cuda_softmax_grad_f32": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32]),
    "bwpp_cuda_reduce_sum_f32": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32, C.c_int]),
    "bwpp_cuda_broadcast_f32": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32, C.c_int]),
    "bwpp_cuda_cast_f32_bf16": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32]),
    "bwpp_cuda_comm_unique_id": (_i32, [_vp]),
    "bwpp_cuda_comm_create": (_i32, [C.POINTER(_vp), _vp, _i32, _i32, _i32]),
    "bwpp_cuda_comm_allreduce_sum_f32": (_i32, [_vp, _vp, _sz, _vp]),
    "bwpp_cuda_comm_destroy": (_i32, [_vp]),
    "bwpp_cuda_comm_create_timeout": (_i32, [C.POINTER(_vp), _vp, _i32, _i32, _i32, _u32]),
    "bwpp_cuda_comm_set_timeout": (_i32, [_vp, _u32]),
    "bwpp_cuda_comm_wait": (_i32, [_vp]),
    "bwpp_cuda_comm_aborted": (_i32, [_vp]),
    "bwpp_cuda_comm_watch": (_i32, [_vp, _vp, _vp, _vp, _u32]),
    "bwpp_cuda_matmul_f32_dist": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _vp,
                                         _i32, _i32]),
    "bwpp_cuda_tiny_model_create": (_i32, [_vp, C.POINTER(TinyModelConfig), _u64, C.POINTER(_vp)]),
    "bwpp_cuda_tiny_model_destroy": (_i32, [_vp]),
    "bwpp_cuda_tiny_model_param_count": (_sz, [_vp]),
    "bwpp_cuda_tiny_model_get": (_i32, [_vp, _vp, _vp]),
    "bwpp_cuda_tiny_model_set_params": (_i32, [_vp, _vp]),
    "bwpp_cuda_tiny_model_input_grad": (_i32, [_vp, _vp]),
    "bwpp_cuda_attention_fwd_lse_bf16": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _f32, _i32,
                                                _vp, _u32, _vp]),
    "bwpp_cuda_attention_bwd_bf16": (_i32, [_vp, _vp, _vp, _vp, _u32, _vp, _u32, _vp, _u32, _vp,
                                            _u32, _u32, _u32, _f32, _i32, _vp, _vp, _vp, _u32]),
    "bwpp_cuda_tiny_model_step": (_i32, [_vp, _vp, _vp, _f32, _vp, _vp]),
    "bwpp_cuda_matmul_f32": (None, [_vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _vp, _i32, _i32]),
    "bwpp_cuda_softmax_f32": (None, [_vp, _vp, _u32, _u32, _u32]),
    "bwpp_cuda_rmsnorm_f32": (None, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _f32]),
    "bwpp_cuda_attention_f32": (None, [_vp, _vp, _vp, _vp] + [_u32] * 8),
    "bwpp_cuda_reduce_max_mask_f32": (None, [_vp, _vp, _u32, _u32, _i32]),
    "bwpp_cuda_reduce_max_grad_f32": (None, [_vp, _vp, _vp, _u32, _u32, _i32]),
    "bwpp_cuda_last_status": (_i32, []),
    "bwpp_cuda_dispatch_matmul": (_i32, [_vp, _vp, _vp, _vp, _vp, MatmulParams, _cp]),
    "bwpp_cuda_dispatch_softmax": (_i32, [_vp, _vp, _vp, SoftmaxParams, _cp]),
    "bwpp_cuda_dispatch_rmsnorm": (_i32, [_vp, _vp, _vp, _vp, _vp, RmsnormParams, _cp]),
    "bwpp_cuda_dispatch_attention": (_i32, [_vp, _vp, _vp, _vp, _vp, AttentionParams, _cp]),
    # f16 variants (half ABI)
    "bwpp_cuda_matmul_f16": (_i32, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _u32, _vp, _i32, _i32]),
    "bwpp_cuda_attention_f16": (_i32, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _u32, _u32, _f32, _i32]),
    "bwpp_cuda_softmax_f16": (_i32, [_vp, _vp, _vp, _u32, _u32, _u32]),
    "bwpp_cuda_rmsnorm_f16": (_i32, [_vp, _vp, _vp, _vp, _vp, _u32, _u32, _u32, _f32]),
    "bwpp_cuda_cast_f16_f32": (_i32, [_vp, _vp, _vp, C.c_size_t]),
    "bwpp_cuda_cast_f32_f16": (_i32, [_vp, _vp, _vp, C.c_size_t]),
    "bwpp_cuda_dispatch_matmul_f16": (_i32, [_vp, _vp, _vp, _vp, _vp, MatmulParams, _cp]),
    "bwpp_cuda_dispatch_softmax_f16": (_i32, [_vp, _vp, _vp, SoftmaxParams, _cp]),
    "bwpp_cuda_dispatch_rmsnorm_f16": (_i32, [_vp, _vp, _vp, _vp, _vp, RmsnormParams, _cp]),
    "bwpp_cuda_dispatch_attention_f16": (_i32, [_vp, _vp, _vp, _vp, _vp, AttentionParams, _cp]),
    # launch-plan executor
    "bwpp_cuda_plan_create": (_i32, [_vp, _cp, _cp, _cp, _cp, C.POINTER(_vp)]),
    "bwpp_cuda_plan_create_launch": (_i32, [_vp, _cp, _cp, C.POINTER(_vp)]),
    "bwpp_cuda_plan_last_error": (_cp, []),
    "bwpp_cuda_plan_describe": (_i32, [_vp, C.c_char_p, C.c_size_t]),
    "bwpp_cuda_plan_find": (_i32, [_vp, _cp]),
    "bwpp_cuda_plan_value_count": (_i32, [_vp]),
    "bwpp_cuda_plan_value_info": (_i32, [_vp, _i32, C.POINTER(_i32), C.POINTER(_i32),
                                         C.POINTER(C.c_int64), C.POINTER(_i32)]),
    "bwpp_cuda_plan_bind": (_i32, [_vp, _i32, _vp]),
    "bwpp_cuda_plan_value_ptr": (_vp, [_vp, _i32]),
    "bwpp_cuda_plan_run": (_i32, [_vp]),
    "bwpp_cuda_plan_launches": (C.c_size_t, [_vp]),
    "bwpp_cuda_plan_destroy": (_i32, [_vp]),
}

_lib = None


def header_symbols(path: str = HEADER_PATH) -> list[str]:
    """Function names declared in include/bwpp_cuda.h."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(bwpp_cuda_\w+)\s*\(", text)))


def load(path: str = LIB_PATH) -> C.CDLL:
    """Loads the CUDA runtime library; raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        raise ImportError(
            f"{path} is missing: build it with `make -C bluewolf-plus-plus_b200` "
            "(or __graft_entry__.build()); there is no CPU fallback")
    lib = C.CDLL(path)
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def status_string(status: int) -> str:
    return load().bwpp_cuda_status_string(status).decode()


def _ptr(t):
    """Device / host address of a torch tensor, numpy array or int (None -> NULL)."""
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if hasattr(t, "data_ptr"):
        return t.data_ptr()
    if hasattr(t, "ctypes"):
        return t.ctypes.data
    raise TypeError(type(t))


class Ctx:
    """A BwppCudaCtx bound to one device and stream (torch's current stream by default)."""

    def __init__(self, device: int = 0, stream=None):
        self.lib = load()
        if stream is None:
            import torch
            stream = torch.cuda.current_stream(device).cuda_stream
        handle = C.c_void_p()
        rc = self.lib.bwpp_cuda_ctx_create(C.byref(handle), device, stream)
        if rc != OK:
            raise BwppError(rc, f"ctx_create(device={device}) failed: {status_string(rc)}")
        self.handle = handle
        self.device = device

    def close(self):
        if self.handle:
            self.lib.bwpp_cuda_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, rc: int, what: str = ""):
        if rc != OK:
            msg = self.lib.bwpp_cuda_ctx_last_error(self.handle).decode()
            raise BwppError(rc, f"{what}: {msg}")

    def sync(self):
        self.check(self.lib.bwpp_cuda_sync(self.handle), "sync")

    def set_stream(self, stream):
        self.check(self.lib.bwpp_cuda_ctx_set_stream(self.handle, stream), "set_stream")

    def set_workspace(self, ptr, nbytes):
        self.check(self.lib.bwpp_cuda_ctx_set_workspace(self.handle, _ptr(ptr), nbytes), "set_workspace")

    # ---- ops (device tensors) -----------------------------------------
    def matmul_bf16(self, a, b, c, M, N, K, lda, ldb, ldc, bias=None, silu=0, add=0):
        self.check(self.lib.bwpp_cuda_matmul_bf16(self.handle, _ptr(a), _ptr(b), _ptr(c), M, N, K,
                                                  lda, ldb, ldc, _ptr(bias), int(silu), int(add)),
                   "matmul_bf16")

    def gemm_ex(self, a, b, c, M, N, K, lda, ldb, ldc, a_mn=0, b_mn=1, out_bf16=0, silu=0,
                bias=None, residual=None, ldr=0):
        p = GemmParams(M, N, K, lda, ldb, ldc, ldr, int(a_mn), int(b_mn), int(out_bf16), int(silu),
                       _ptr(bias), _ptr(residual))
        self.check(self.lib.bwpp_cuda_gemm_bf16_ex(self.handle, _ptr(a), _ptr(b), _ptr(c), C.byref(p)),
                   "gemm_bf16_ex")

    def attention_bf16(self, q, k, v, o, B, H, Sq, Skv, D, scale, causal):
        self.check(self.lib.bwpp_cuda_attention_bf16(self.handle, _ptr(q), _ptr(k), _ptr(v), _ptr(o),
                                                     B, H, Sq, Skv, D, float(scale), int(causal)),
                   "attention_bf16")

    def rmsnorm_fwd(self, x, y, gamma, beta, rows, cols, ld, eps):
        self.check(self.lib.bwpp_cuda_rmsnorm_fwd_f32(self.handle, _ptr(x), _ptr(y), _ptr(gamma),
                                                      _ptr(beta), rows, cols, ld, eps), "rmsnorm_fwd")

    def layernorm_fwd(self, x, y, gamma, beta, rows, cols, ld, eps):
        self.check(self.lib.bwpp_cuda_layernorm_fwd_f32(self.handle, _ptr(x), _ptr(y), _ptr(gamma),
                                                        _ptr(beta), rows, cols, ld, eps), "layernorm_fwd")

    def rmsnorm_bwd(self, x, gamma, dy, dx, dgamma, dbeta, rows, cols, ld, eps):
        self.check(self.lib.bwpp_cuda_rmsnorm_bwd_f32(self.handle, _ptr(x), _ptr(gamma), _ptr(dy), _ptr(dx),
                                                      _ptr(dgamma), _ptr(dbeta), rows, cols, ld, eps),
                   "rmsnorm_bwd")

    def layernorm_bwd(self, x, gamma, dy, dx, dgamma, dbeta, rows, cols, ld, eps):
        self.check(self.lib.bwpp_cuda_layernorm_bwd_f32(self.handle, _ptr(x), _ptr(gamma), _ptr(dy), _ptr(dx),
                                                        _ptr(dgamma), _ptr(dbeta), rows, cols, ld, eps),
                   "layernorm_bwd")

    def reduce_max_fwd(self, x, maxv, argmax, rows, cols, ld):
        self.check(self.lib.bwpp_cuda_reduce_max_fwd_f32(self.handle, _ptr(x), _ptr(maxv), _ptr(argmax),
                                                         rows, cols, ld), "reduce_max_fwd")

    def reduce_max_bwd(self, argmax, dy, dx, rows, cols, ld):
        self.check(self.lib.bwpp_cuda_reduce_max_bwd_f32(self.handle, _ptr(argmax), _ptr(dy), _ptr(dx),
                                                         rows, cols, ld), "reduce_max_bwd")

    def reduce_max_mask(self, x, mask, rows, cols, axis):
        self.check(self.lib.bwpp_cuda_reduce_max_mask_ex(self.handle, _ptr(x), _ptr(mask), rows, cols, axis),
                   "reduce_max_mask")

    def reduce_max_grad(self, mask, dy, dx, rows, cols, axis):
        self.check(self.lib.bwpp_cuda_reduce_max_grad_ex(self.handle, _ptr(mask), _ptr(dy), _ptr(dx),
                                                         rows, cols, axis), "reduce_max_grad")

    def softmax_fwd(self, x, y, rows, cols, ld):
        self.check(self.lib.bwpp_cuda_softmax_fwd_f32(self.handle, _ptr(x), _ptr(y), rows, cols, ld),
                   "softmax_fwd")

    # f16 variants (half ABI): tensors hold IEEE half (torch.float16)
    def matmul_f16(self, a, b, c, M, N, K, lda, ldb, ldc, bias=None, silu=0, add=0):
        self.check(self.lib.bwpp_cuda_matmul_f16(self.handle, _ptr(a), _ptr(b), _ptr(c), M, N, K, lda,
                                                 ldb, ldc, _ptr(bias), int(silu), int(add)),
                   "matmul_f16")

    def attention_f16(self, q, k, v, o, B, H, Sq, Skv, D, scale, causal):
        self.check(self.lib.bwpp_cuda_attention_f16(self.handle, _ptr(q), _ptr(k), _ptr(v), _ptr(o),
                                                    B, H, Sq, Skv, D, float(scale), int(causal)),
                   "attention_f16")

    def softmax_f16(self, x, y, rows, cols, ld):
        self.check(self.lib.bwpp_cuda_softmax_f16(self.handle, _ptr(x), _ptr(y), rows, cols, ld),
                   "softmax_f16")

    def rmsnorm_f16(self, x, y, gamma, beta, rows, cols, ld, eps):
        self.check(self.lib.bwpp_cuda_rmsnorm_f16(self.handle, _ptr(x), _ptr(y), _ptr(gamma), _ptr(beta),
                                                  rows, cols, ld, float(eps)), "rmsnorm_f16")

    # autodiff-internal ops (fp32)
    def silu_grad(self, x, dy, dx, n):
        self.check(self.lib.bwpp_cuda_silu_grad_f32(self.handle, _ptr(x), _ptr(dy), _ptr(dx), n),
                   "silu_grad")

    def softmax_grad(self, y, dy, dx, rows, cols, ld):
        self.check(self.lib.bwpp_cuda_softmax_grad_f32(self.handle, _ptr(y), _ptr(dy), _ptr(dx), rows,
                                                       cols, ld), "softmax_grad")

    def reduce_sum(self, x, out, rows, cols, ld, axis):
        self.check(self.lib.bwpp_cuda_reduce_sum_f32(self.handle, _ptr(x), _ptr(out), rows, cols, ld,
                                                     axis), "reduce_sum")

    def broadcast(self, src, dst, rows, cols, ld, axis):
        self.check(self.lib.bwpp_cuda_broadcast_f32(self.handle, _ptr(src), _ptr(dst), rows, cols, ld,
                                                    axis), "broadcast")

    def cast_f32_bf16(self, src, dst, rows, cols, ld_src):
        self.check(self.lib.bwpp_cuda_cast_f32_bf16(self.handle, _ptr(src), _ptr(dst), rows, cols, ld_src),
                   "cast_f32_bf16")


class Plan:
    """A graph of the reference compiler lowered onto the CUDA kernels: the
    launch plan `bwppc --target cuda --dims ...` writes (pass its text as
    graph_dot; mem_plan and dims are then unused), or its --dot / --grad-dot
    dump and optionally its --mem-plan dump, lowered here.

        plan = Plan(ctx, open("g.dot").read(), open("m.txt").read(), {"T": 128, "D": 256})
        plan.bind("x", x_tensor); ...; plan.run(); y = plan.tensor("out")

    ctx=None parses and lowers only (describe() works without a GPU)."""

    DTYPES = {0: "float16", 1: "bfloat16", 2: "float32"}

    def __init__(self, ctx, graph_dot: str, mem_plan: str | None = None, dims: dict | None = None,
                 options: str | None = None):
        self.lib = load()
        self.ctx = ctx
        spec = ",".join(f"{k}={int(v)}" for k, v in (dims or {}).items())
        h = C.c_void_p()
        if graph_dot.lstrip().startswith("// BW++ CUDA launch plan"):
            # the output of `bwppc --target cuda` (dims are bound in it)
            rc = self.lib.bwpp_cuda_plan_create_launch(ctx.handle if ctx is not None else None,
                                                       graph_dot.encode(),
                                                       options.encode() if options else None, C.byref(h))
        else:
            rc = self.lib.bwpp_cuda_plan_create(ctx.handle if ctx is not None else None, graph_dot.encode(),
                                                mem_plan.encode() if mem_plan else None, spec.encode(),
                                                options.encode() if options else None, C.byref(h))
        if rc != 0:
            raise RuntimeError(f"plan_create: {status_string(rc)}: "
                               f"{self.lib.bwpp_cuda_plan_last_error().decode()}")
        self.handle = h
        self._bound = {}

    def describe(self) -> str:
        n = self.lib.bwpp_cuda_plan_describe(self.handle, None, 0)
        buf = C.create_string_buffer(n)
        self.lib.bwpp_cuda_plan_describe(self.handle, buf, n)
        return buf.value.decode()

    def steps(self) -> list:
        return [ln for ln in self.describe().splitlines() if ln and not ln.startswith("arena")]

    def id(self, name_or_id) -> int:
        if isinstance(name_or_id, int):
            return name_or_id
        vid = self.lib.bwpp_cuda_plan_find(self.handle, name_or_id.encode())
        if vid < 0:
            raise KeyError(name_or_id)
        return vid

    def info(self, name_or_id) -> dict:
        vid = self.id(name_or_id)
        dt, rank, flags = C.c_int(), C.c_int(), C.c_int()
        dims = (C.c_int64 * 8)()
        rc = self.lib.bwpp_cuda_plan_value_info(self.handle, vid, C.byref(dt), C.byref(rank), dims,
                                                C.byref(flags))
        if rc != 0:
            raise KeyError(name_or_id)
        return {"id": vid, "dtype": self.DTYPES[dt.value], "shape": tuple(dims[:rank.value]),
                "input": bool(flags.value & 1), "output": bool(flags.value & 2),
                "held": bool(flags.value & 4)}

    def values(self) -> list:
        out = []
        for i in range(self.lib.bwpp_cuda_plan_value_count(self.handle)):
            try:
                out.append(self.info(i))
            except KeyError:
                pass
        return out

    def bind(self, name_or_id, tensor):
        vid = self.id(name_or_id)
        self._bound[vid] = tensor  # kept alive while the plan may read it
        rc = self.lib.bwpp_cuda_plan_bind(self.handle, vid, _ptr(tensor))
        if rc != 0:
            raise RuntimeError(f"plan_bind({name_or_id}): {status_string(rc)}")

    def run(self):
        rc = self.lib.bwpp_cuda_plan_run(self.handle)
        if self.ctx is None:
            raise RuntimeError("plan_run: the plan was created without a context")
        self.ctx.check(rc, "plan_run")

    @property
    def launches(self) -> int:
        return int(self.lib.bwpp_cuda_plan_launches(self.handle))

    def tensor(self, name_or_id):
        """A torch view of a value held in the plan's memory (valid until close)."""
        import torch
        meta = self.info(name_or_id)
        ptr = self.lib.bwpp_cuda_plan_value_ptr(self.handle, meta["id"])
        if not ptr:
            raise RuntimeError(f"{name_or_id} is not materialised")
        dtype = getattr(torch, meta["dtype"])
        n = 1
        for d in meta["shape"]:
            n *= d
        esz = torch.empty(0, dtype=dtype).element_size()
        return _cuda_view(ptr, n * esz, self.ctx.device if self.ctx is not None else 0).view(dtype) \
            .reshape(meta["shape"])

    def close(self):
        if getattr(self, "handle", None):
            self.lib.bwpp_cuda_plan_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _cuda_view(ptr: int, nbytes: int, device: int):
    """uint8 torch tensor aliasing nbytes of device memory at ptr (no copy)."""
    import torch

    class _Arr:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                    "version": 3}
    with torch.cuda.device(device):
        return torch.as_tensor(_Arr(), device=f"cuda:{device}")


class TinyModel:
    """The tiny_model training step (bwpp_cuda_tiny_model_*) on one Ctx."""

    def __init__(self, ctx: "Ctx", layers, d_model, heads, ffn, batch, seq, eps=1e-5, seed=1):
        self.ctx, self.lib = ctx, ctx.lib
        self.cfg = TinyModelConfig(layers, d_model, heads, 128, ffn, batch, seq, eps)
        h = C.c_void_p()
        ctx.check(self.lib.bwpp_cuda_tiny_model_create(ctx.handle, C.byref(self.cfg), seed, C.byref(h)),
                  "tiny_model_create")
        self.handle = h
        self.count = self.lib.bwpp_cuda_tiny_model_param_count(h)

    def step(self, x, target, lr=0.0, comm=None, loss_out=None):
        self.ctx.check(self.lib.bwpp_cuda_tiny_model_step(self.handle, _ptr(x), _ptr(target), float(lr),
                                                          comm, _ptr(loss_out)), "tiny_model_step")

    def get(self, params_out=None, grads_out=None):
        self.ctx.check(self.lib.bwpp_cuda_tiny_model_get(self.handle, _ptr(params_out), _ptr(grads_out)),
                       "tiny_model_get")

    def input_grad(self, dx_out):
        self.ctx.check(self.lib.bwpp_cuda_tiny_model_input_grad(self.handle, _ptr(dx_out)),
                       "tiny_model_input_grad")

    def set_params(self, params):
        self.ctx.check(self.lib.bwpp_cuda_tiny_model_set_params(self.handle, _ptr(params)),
                       "tiny_model_set_params")

    def close(self):
        if self.handle:
            self.lib.bwpp_cuda_tiny_model_destroy(self.handle)
            self.handle = None


# ---- CPU-signature mirrors (host or device pointers, synchronous) ---------

def _mirror_check(what):
    rc = load().bwpp_cuda_last_status()
    if rc != OK:
        raise BwppError(rc, f"{what}: {status_string(rc)}")


def matmul_f32(a, b, c, M, N, K, lda, ldb, ldc, bias, apply_silu, apply_bias):
    load().bwpp_cuda_matmul_f32(_ptr(a), _ptr(b), _ptr(c), M, N, K, lda, ldb, ldc, _ptr(bias),
                                int(apply_silu), int(apply_bias))
    _mirror_check("bwpp_cuda_matmul_f32")


def matmul_f32_dist(comm, a, b, c, M, N, K, lda, ldb, ldc, bias, apply_silu, apply_bias):
    """bwpp_cuda_matmul_f32_dist: this rank's rows of a / c, all of b and bias (host memory)."""
    rc = load().bwpp_cuda_matmul_f32_dist(comm, _ptr(a), _ptr(b), _ptr(c), M, N, K, lda, ldb, ldc,
                                          _ptr(bias), int(apply_silu), int(apply_bias))
    if rc != OK:
        raise BwppError(rc, f"bwpp_cuda_matmul_f32_dist: {status_string(rc)}")


def softmax_f32(x, y, rows, cols, ld):
    load().bwpp_cuda_softmax_f32(_ptr(x), _ptr(y), rows, cols, ld)
    _mirror_check("bwpp_cuda_softmax_f32")


def rmsnorm_f32(x, y, gamma, beta, rows, cols, ld, eps):
    load().bwpp_cuda_rmsnorm_f32(_ptr(x), _ptr(y), _ptr(gamma), _ptr(beta), rows, cols, ld, eps)
    _mirror_check("bwpp_cuda_rmsnorm_f32")


def attention_f32(q, k, v, o, M, N, K, D, ldq, ldk, ldv, ldo):
    load().bwpp_cuda_attention_f32(_ptr(q), _ptr(k), _ptr(v), _ptr(o), M, N, K, D, ldq, ldk, ldv, ldo)
    _mirror_check("bwpp_cuda_attention_f32")


def reduce_max_mask_f32(x, mask, rows, cols, axis):
    load().bwpp_cuda_reduce_max_mask_f32(_ptr(x), _ptr(mask), rows, cols, axis)
    _mirror_check("bwpp_cuda_reduce_max_mask_f32")


def reduce_max_grad_f32(mask, dy, dx, rows, cols, axis):
    load().bwpp_cuda_reduce_max_grad_f32(_ptr(mask), _ptr(dy), _ptr(dx), rows, cols, axis)
    _mirror_check("bwpp_cuda_reduce_max_grad_f32")
