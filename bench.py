#!/usr/bin/env python3
"""BW++ B200 benchmark.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload gemm|attention|attention_causal|rmsnorm_fwd|
                                rmsnorm_bwd|layernorm_fwd|layernorm_bwd|
                                reduce_max_fwd|reduce_max_bwd|softmax_fwd|
                                softmax_grad|silu_grad|reduce_sum_rows|
                                reduce_sum_cols|broadcast_rows|gemm_f16|
                                attention_f16|attention_causal_f16|attention_bwd|
                                tiny_model|plan_tiny_model]

Default workload (the headline): fused matmul + bias +
SiLU, X[8192x4096] bf16 * W[4096x11008] bf16 + b[11008], fp32 out, rows of X
split over the N ranks (one process per GPU, torchrun), no collective on the
data path.  The other workloads are BASELINE configs[2] / configs[3] kernels.

One JSON line on rank 0:
  value         whole-job throughput, inputs resident in HBM, CUDA events on
                the launching stream around each step, max over ranks
  e2e           the same metric through the reference-facing C ABI mirror
                (bwpp_cuda_*_f32 with pinned HOST buffers: host->device copies,
                the kernel and the device->host copy of the result are timed)
  roofline      the dominant kernel against MEASURED_PEAKS.json
  cpu_baseline  the reference's own CPU code (oracle/_ref, built from the
                reference sources) on a bounded row sample, rank 0 at N=1
  clocks        NVML samples taken while the timed steps execute

--impl reference times the reference's own CPU implementation on the host
cores (rank 0 only; other ranks exit 0), same metric / unit / config.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
for p in (os.path.join(ROOT, "bluewolf-plus-plus_b200"), os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

METRIC = "TFLOP/s (GEMM, attention) & HBM GB/s (norms) per B200 at 1/2/4/8 GPUs"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
L2_FLUSH_BYTES = 256 << 20


# ---------------------------------------------------------------------------
# helpers
# ---------------------------------------------------------------------------

def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(path))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", d["bf16_tflops"])), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def profile_traffic(name):
    """dram bytes per launch recorded in profiles/<name>.md (from an ncu capture)."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    try:
        for line in open(path):
            if line.strip().startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1].strip().split()[0])
    except OSError:
        pass
    return None


from bwpp.dist import comm_from_process_group, max_over_ranks, split_rows  # noqa: E402


class ClockSampler:
    """NVML SM clock / throttle-reason samples; poll() while the timed work runs."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x2: "applications_clocks_setting", 0x1: "gpu_idle"}

    def __init__(self, device):
        self.samples, self.reasons, self.max_mhz, self.h = [], set(), None, None
        try:
            import pynvml as N
            import torch
            N.nvmlInit()
            self.N = N
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            try:
                self.h = N.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
            except Exception:
                self.h = N.nvmlDeviceGetHandleByUUID("GPU-" + uuid)
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(self.h, N.NVML_CLOCK_SM)
        except Exception:
            self.h = None
        self.last = 0.0

    def poll(self, force=False):
        if self.h is None:
            return
        now = time.perf_counter()
        if not force and now - self.last < 0.004:
            return
        self.last = now
        N = self.N
        try:
            self.samples.append(N.nvmlDeviceGetClockInfo(self.h, N.NVML_CLOCK_SM))
            try:
                bits = N.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except AttributeError:
                bits = N.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
            for b, name in self.REASONS.items():
                if bits & b and b != 0x1:
                    self.reasons.add(name)
        except Exception:
            pass

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": float(np.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------

class Workload:
    """One step = one pass of the hot path over this rank's shard."""
    unit = "TFLOP/s"
    bound = "tensor"
    dtype = "bf16"

    def __init__(self, rank, world, torch, bwpp, ctx):
        self.rank, self.world, self.torch, self.bwpp, self.ctx = rank, world, torch, bwpp, ctx

    def work_per_step(self):           # algorithmic FLOP or bytes of this rank per step
        raise NotImplementedError

    def total_work_per_step(self):     # all ranks
        raise NotImplementedError

    def scale(self, work, seconds):
        return work / seconds / (1e12 if self.unit == "TFLOP/s" else 1e9)


class GemmWorkload(Workload):
    """X[8192x4096] W[4096x11008] + b, SiLU, fp32 out."""
    M, K, N = 8192, 4096, 11008
    kernel = "gemm_tc_kernel"
    profile = "gemm_tc_kernel_config2"

    def setup(self):
        t = self.torch
        self.r0, self.r1 = split_rows(self.M, self.rank, self.world)
        self.m = self.r1 - self.r0
        g = t.Generator(device="cuda").manual_seed(2000)
        x = t.randn(self.M, self.K, device="cuda", generator=g) * 0.02
        self.x = x[self.r0:self.r1].to(t.bfloat16).contiguous()
        del x
        self.w = (t.randn(self.K, self.N, device="cuda", generator=g) * 0.02).to(t.bfloat16)
        self.b = t.rand(self.N, device="cuda", generator=g) * 0.2 - 0.1
        self.c = t.empty(self.m, self.N, device="cuda")

    def step(self):
        self.ctx.matmul_bf16(self.x, self.w, self.c, self.m, self.N, self.K, self.K, self.N, self.N,
                             self.b, 1, 1)
        return 1

    def work_per_step(self):
        return 2.0 * self.m * self.N * self.K

    def total_work_per_step(self):
        return 2.0 * self.M * self.N * self.K

    def config(self):
        return {"workload": "fused matmul+bias+SiLU (BASELINE configs[1], examples/matmul_add_silu)",
                "M": self.M, "K": self.K, "N": self.N, "rows_per_gpu": self.m,
                "inputs": "X,W ~ N(0,0.02) bf16, b ~ U(-0.1,0.1) fp32, out fp32",
                "parallelism": f"rows of X over {self.world} GPU(s), W replicated, no collective",
                "l2": "256 MiB written between timed steps (flush)"}

    # e2e through the CPU-signature mirror with pinned host buffers; on N GPUs
    # its multi-GPU form, where each rank uploads 1/N of W and NCCL
    # all-gathers the bf16 W over NVLink
    def setup_e2e(self):
        t = self.torch
        self.ha = self.x.float().cpu().pin_memory()
        self.hb = self.w.float().cpu().pin_memory()
        self.hbias = self.b.cpu().pin_memory()
        self.hc = t.empty(self.m, self.N, dtype=t.float32).pin_memory()
        self.h2d = (self.m * self.K + self.K * self.N + self.N) * 4
        self.d2h = self.m * self.N * 4
        if self.world > 1:
            import torch.distributed as dist
            self.comm = comm_from_process_group(self.bwpp.load(), self.rank, self.world,
                                                t.cuda.current_device(), dist)
            kc = -(-self.K // self.world)
            k0 = min(self.rank * kc, self.K)
            k1 = min(k0 + kc, self.K)
            self.h2d = (self.m * self.K + (k1 - k0) * self.N + self.N) * 4
            self.e2e_api = ("bwpp_cuda_matmul_f32_dist (the f32 mirror across the ranks): pinned host "
                            "A rows, 1/N of W's K rows and b in, NCCL all-gather of bf16 W, C rows out")

    def step_e2e(self):
        if self.world > 1:
            self.bwpp.matmul_f32_dist(self.comm, self.ha, self.hb, self.hc, self.m, self.N, self.K, self.K,
                                      self.N, self.N, self.hbias, 1, 1)
            return
        self.bwpp.matmul_f32(self.ha, self.hb, self.hc, self.m, self.N, self.K, self.K, self.N, self.N,
                             self.hbias, 1, 1)

    # reference CPU code on a bounded row sample
    def cpu_sample(self, lib, threads):
        import oracle as O
        rows = max(threads, 4)
        if not hasattr(self, "cpu_a"):
            rng = np.random.default_rng(2000)
            self.cpu_a = (0.02 * rng.standard_normal((rows, self.K))).astype(np.float32)
            self.cpu_b = (0.02 * rng.standard_normal((self.K, self.N))).astype(np.float32)
            self.cpu_bias = rng.uniform(-0.1, 0.1, self.N).astype(np.float32)
            self.cpu_c = np.zeros((rows, self.N), np.float32)
        t0 = time.perf_counter()
        O.run_rows_threaded(lambda r0, r1: O.ref_matmul_rows(lib, self.cpu_a, self.cpu_b, self.cpu_c,
                                                             self.cpu_bias, 1, 1, r0, r1), rows, threads)
        dt = time.perf_counter() - t0
        return 2.0 * rows * self.N * self.K, dt, f"{rows} of 8192 rows x all 11008 columns, K=4096, fp32, row-split over {threads} threads"


class GemmF16Workload(GemmWorkload):
    """configs[1] shapes through the half ABI (bwpp_cuda_matmul_f16): f16 X, W,
    b and C, fp32 accumulation."""
    dtype = "f16"
    profile = "gemm_tc_kernel_f16_config2"
    e2e_api = "bwpp_cuda_matmul_f16; pinned host f16 X, W, b copied in and C copied out every step"

    def setup(self):
        super().setup()
        t = self.torch
        self.x = self.x.to(t.float16)
        self.w = self.w.to(t.float16)
        self.b = self.b.to(t.float16)
        self.c = t.empty(self.m, self.N, dtype=t.float16, device="cuda")

    def step(self):
        self.ctx.matmul_f16(self.x, self.w, self.c, self.m, self.N, self.K, self.K, self.N, self.N,
                            self.b, 1, 1)
        return 2  # bias widening + GEMM

    def config(self):
        cfg = super().config()
        cfg["workload"] = "fused matmul+bias+SiLU, half ABI (configs[1] shapes)"
        cfg["inputs"] = "X,W ~ N(0,0.02) f16, b ~ U(-0.1,0.1) f16, out f16"
        return cfg

    def setup_e2e(self):
        t = self.torch
        self.ha, self.hb, self.hbias = (u.cpu().pin_memory() for u in (self.x, self.w, self.b))
        self.hc = t.empty(self.m, self.N, dtype=t.float16).pin_memory()
        self.h2d = (self.m * self.K + self.K * self.N + self.N) * 2
        self.d2h = self.m * self.N * 2

    def step_e2e(self):
        self.x.copy_(self.ha, non_blocking=True)
        self.w.copy_(self.hb, non_blocking=True)
        self.b.copy_(self.hbias, non_blocking=True)
        self.step()
        self.hc.copy_(self.c, non_blocking=True)
        self.torch.cuda.synchronize()

    def cpu_sample(self, lib, threads):
        return None


class AttentionWorkload(Workload):
    """B=8 H=32 S=4096 d=128, bf16 in, fp32 out; heads over ranks."""
    B, H, S, D = 8, 32, 4096, 128
    kernel = "attention"
    profile = "attention_tc_kernel_config4"

    def __init__(self, *a, causal=False):
        super().__init__(*a)
        self.causal = causal

    def setup(self):
        t = self.torch
        self.h0, self.h1 = split_rows(self.B * self.H, self.rank, self.world)
        self.nh = self.h1 - self.h0
        g = t.Generator(device="cuda").manual_seed(4000 + self.h0)
        self.q, self.k, self.v = (t.randn(self.nh, self.S, self.D, device="cuda", generator=g).to(t.bfloat16)
                                  for _ in range(3))
        self.o = t.empty(self.nh, self.S, self.D, device="cuda")
        # kernels per call: a non-causal launch whose last round of items (256
        # query rows of one head, one CTA per SM) is at most half full runs
        # that round as a second, split launch (attention_tc.cu)
        sms = t.cuda.get_device_properties(t.cuda.current_device()).multi_processor_count
        items = -(-self.S // 256) * self.nh
        self.kernels = 2 if (not self.causal and items > sms and 0 < items % sms <= sms // 2
                             and -(-self.S // 128) >= 2) else 1

    def step(self):
        self.ctx.attention_bf16(self.q, self.k, self.v, self.o, 1, self.nh, self.S, self.S, self.D,
                                self.D ** -0.5, int(self.causal))
        return self.kernels

    def flops_per_head(self):
        S, D = self.S, self.D
        return 4.0 * D * S * (S + 1) / 2 if self.causal else 4.0 * S * S * D

    def work_per_step(self):
        return self.nh * self.flops_per_head()

    def total_work_per_step(self):
        return self.B * self.H * self.flops_per_head()

    def config(self):
        return {"workload": f"attention {'causal' if self.causal else 'non-causal'} (BASELINE configs[3])",
                "B": self.B, "H": self.H, "S": self.S, "D": self.D, "heads_per_gpu": self.nh,
                "parallelism": f"batch x head over {self.world} GPU(s), no collective",
                "l2": "256 MiB written between timed steps (flush)"}

    def setup_e2e(self):
        self.hq, self.hk, self.hv = (t.float().cpu().pin_memory() for t in (self.q, self.k, self.v))
        self.ho = self.torch.empty(self.nh, self.S, self.D).pin_memory()
        self.h2d = 3 * self.nh * self.S * self.D * 4
        self.d2h = self.nh * self.S * self.D * 4

    def step_e2e(self):
        if self.causal:
            raise NotImplementedError
        for h in range(self.nh):  # the reference's 2-D entry point is one head at a time
            self.bwpp.attention_f32(self.hq[h], self.hk[h], self.hv[h], self.ho[h], self.S, self.S,
                                    self.D, self.D, self.D, self.D, self.D, self.D)

    def cpu_sample(self, lib, threads):
        import oracle as O
        rows = max(threads, 4)
        rng = np.random.default_rng(4000)
        q = rng.standard_normal((rows, self.D)).astype(np.float32) * np.float32(self.D ** -0.5)
        k = rng.standard_normal((self.S, self.D)).astype(np.float32)
        v = rng.standard_normal((self.S, self.D)).astype(np.float32)
        o = np.zeros((rows, self.D), np.float32)
        import ctypes as C
        fp = C.POINTER(C.c_float)

        def part(r0, r1):
            for r in range(r0, r1):
                n = (r * (self.S // rows) + 1) if self.causal else self.S
                lib.attention_f32(C.cast(C.c_void_p(q.ctypes.data + r * self.D * 4), fp),
                                  k.ctypes.data_as(fp), v.ctypes.data_as(fp),
                                  C.cast(C.c_void_p(o.ctypes.data + r * self.D * 4), fp),
                                  1, n, self.D, self.D, self.D, self.D, self.D, self.D)
        t0 = time.perf_counter()
        O.run_rows_threaded(part, rows, threads)
        dt = time.perf_counter() - t0
        flops = sum(4.0 * self.D * ((r * (self.S // rows) + 1) if self.causal else self.S) for r in range(rows))
        return flops, dt, f"{rows} query rows of one (b,h), S={self.S}, d={self.D}, fp32, {threads} threads"


class AttentionBwdWorkload(Workload):
    """Attention backward of the tiny_model training step (16 x 128
    heads, causal, seq 2048, batch 16 per GPU): bwpp_cuda_attention_bwd_bf16 (delta, then
    the dQ and dK/dV kernels) on token-major bf16 Q, K, V, O, dO; batch over ranks.
    Work is counted as 2.5 x the causal forward's FLOPs (five products of the forward's
    size: S, dP and the dQ / dK / dV products, the recomputed S^T / dP^T not counted)."""
    B, H, S, D = 16, 16, 2048, 128
    kernel = "bwd_dq_kernel + bwd_dkdv_kernel"
    profile = "attention_bwd_tiny_model"
    e2e_api = "bwpp_cuda_attention_bwd_bf16; pinned host Q, K, V, O, dO, lse in, dQ, dK, dV out"

    def setup(self):
        t = self.torch
        self.b0, self.b1 = split_rows(self.B, self.rank, self.world)
        self.nb = self.b1 - self.b0
        T, HD = self.nb * self.S, self.H * self.D
        g = t.Generator(device="cuda").manual_seed(6000 + self.b0)
        self.q, self.k, self.v, self.do = (t.randn(T, HD, device="cuda", generator=g).to(t.bfloat16)
                                           for _ in range(4))
        self.o = t.empty(T, HD, dtype=t.bfloat16, device="cuda")
        self.lse = t.empty(self.nb * self.H * self.S, device="cuda")
        self.dq, self.dk, self.dv = (t.empty(T, HD, dtype=t.bfloat16, device="cuda") for _ in range(3))
        self.lib = self.bwpp.load()
        self.ctx.check(self.lib.bwpp_cuda_attention_fwd_lse_bf16(
            self.ctx.handle, self.q.data_ptr(), self.k.data_ptr(), self.v.data_ptr(), HD, self.nb,
            self.H, self.S, self.D ** -0.5, 1, self.o.data_ptr(), HD, self.lse.data_ptr()), "fwd_lse")
        self.ctx.sync()

    def _bwd(self, q, k, v, o, do, lse, dq, dk, dv):
        HD = self.H * self.D
        self.ctx.check(self.lib.bwpp_cuda_attention_bwd_bf16(
            self.ctx.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), HD, o.data_ptr(), HD,
            do.data_ptr(), HD, lse.data_ptr(), self.nb, self.H, self.S, self.D ** -0.5, 1,
            dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), HD), "attention bwd")

    def step(self):
        self._bwd(self.q, self.k, self.v, self.o, self.do, self.lse, self.dq, self.dk, self.dv)
        return 3  # delta, dQ, dK / dV

    def flops_per_head(self):
        return 2.5 * 4.0 * self.D * self.S * (self.S + 1) / 2

    def work_per_step(self):
        return self.nb * self.H * self.flops_per_head()

    def total_work_per_step(self):
        return self.B * self.H * self.flops_per_head()

    def config(self):
        return {"workload": "attention backward, causal (the tiny_model step's attention, "
                            "BASELINE configs[4])",
                "B": self.B, "H": self.H, "S": self.S, "D": self.D, "batch_per_gpu": self.nb,
                "parallelism": f"batch over {self.world} GPU(s), no collective",
                "flops": "2.5 x the causal forward (S, dP, dQ, dK, dV products)",
                "l2": "256 MiB written between timed steps (flush)"}

    def setup_e2e(self):
        t = self.torch
        self.hin = [u.cpu().pin_memory() for u in (self.q, self.k, self.v, self.o, self.do, self.lse)]
        self.hout = [t.empty_like(u, device="cpu").pin_memory() for u in (self.dq, self.dk, self.dv)]
        self.h2d = sum(u.numel() * u.element_size() for u in self.hin)
        self.d2h = sum(u.numel() * u.element_size() for u in self.hout)

    def step_e2e(self):
        dev = (self.q, self.k, self.v, self.o, self.do, self.lse)
        for d, h in zip(dev, self.hin):
            d.copy_(h, non_blocking=True)
        self.step()
        for h, d in zip(self.hout, (self.dq, self.dk, self.dv)):
            h.copy_(d, non_blocking=True)
        self.torch.cuda.synchronize()

    def cpu_sample(self, lib, threads):
        return None  # the reference has no attention backward


class AttentionF16Workload(AttentionWorkload):
    """configs[3] shapes through the half ABI (bwpp_cuda_attention_f16)."""
    dtype = "f16"
    profile = "attention_tc_kernel_f16_config4"
    e2e_api = "bwpp_cuda_attention_f16; pinned host f16 Q, K, V copied in and O copied out every step"

    def setup(self):
        super().setup()
        t = self.torch
        self.q, self.k, self.v = (u.to(t.float16) for u in (self.q, self.k, self.v))
        self.o = t.empty(self.nh, self.S, self.D, dtype=t.float16, device="cuda")

    def step(self):
        self.ctx.attention_f16(self.q, self.k, self.v, self.o, 1, self.nh, self.S, self.S, self.D,
                               self.D ** -0.5, int(self.causal))
        return 1

    def config(self):
        cfg = super().config()
        cfg["workload"] = cfg["workload"].replace("(BASELINE configs[3])", "half ABI (configs[3] shapes)")
        return cfg

    def setup_e2e(self):
        self.hq, self.hk, self.hv = (u.cpu().pin_memory() for u in (self.q, self.k, self.v))
        self.ho = self.torch.empty(self.nh, self.S, self.D, dtype=self.torch.float16).pin_memory()
        self.h2d = 3 * self.nh * self.S * self.D * 2
        self.d2h = self.nh * self.S * self.D * 2

    def step_e2e(self):
        for dst, src in ((self.q, self.hq), (self.k, self.hk), (self.v, self.hv)):
            dst.copy_(src, non_blocking=True)
        self.step()
        self.ho.copy_(self.o, non_blocking=True)
        self.torch.cuda.synchronize()

    def cpu_sample(self, lib, threads):
        return None


class PlanTinyModelWorkload(Workload):
    """examples/tiny_model.bwpp through the launch-plan executor: the launch
    plan `bwppc --target cuda --dims T=8192,D=1024,H=4096,V=32000` wrote
    (tests/golden/plans/), f16 as the graph declares; one step = one forward
    pass of the graph (24 kernel launches)."""
    T, D, H, V = 8192, 1024, 4096, 32000
    kernel = "plan (tiny_model graph)"
    profile = "plan_tiny_model"
    dtype = "f16"
    e2e_api = "bwpp_cuda_plan_run; pinned host f16 x copied in and the [T,V] probabilities copied out"

    def setup(self):
        t = self.torch
        here = os.path.join(os.path.dirname(os.path.abspath(__file__)), "tests", "golden", "plans")
        name = f"tiny_model@T{self.T}_D{self.D}_H{self.H}_V{self.V}.plan"
        with open(os.path.join(here, name)) as f:
            self.plan = self.bwpp.Plan(self.ctx, f.read())
        g = t.Generator(device="cuda").manual_seed(6000 + self.rank)
        self.inputs = {}
        x_id = self.plan.id("x")
        for v in self.plan.values():
            if not v["input"]:
                continue
            shape = v["shape"]
            # x ~ N(0, 1); weights [in, out] ~ N(0, 1/in); norm gains 1 + N(0, 0.01)
            scale = 1.0 if (len(shape) == 1 or v["id"] == x_id) else shape[0] ** -0.5
            x = t.randn(*shape, device="cuda", generator=g) * (0.1 if len(shape) == 1 else scale)
            if len(shape) == 1:
                x = x + 1.0  # norm gains near 1
            self.inputs[v["id"]] = x.to(t.float16)
            self.plan.bind(v["id"], self.inputs[v["id"]])
        self.x_id = self.plan.id("x")
        self.out_id = [v["id"] for v in self.plan.values() if v["output"]][0]

    def step(self):
        self.plan.run()
        return self.plan.launches

    def flops(self):
        T, D, H, V = self.T, self.D, self.H, self.V
        block = 3 * 2 * T * D * D + 2 * 2 * T * T * D + 2 * T * D * D + 2 * 2 * T * D * H
        return 2 * block + 2 * T * D * V

    def work_per_step(self):
        return float(self.flops())

    def total_work_per_step(self):
        return float(self.flops() * self.world)

    def config(self):
        return {"workload": "examples/tiny_model.bwpp forward from the compiler's launch plan "
                            "(bwppc --target cuda), launch-plan executor",
                "T": self.T, "D": self.D, "H": self.H, "V": self.V,
                "parallelism": f"one replica per GPU ({self.world}), no collective",
                "fusions": "silu and residual-add GEMM epilogues, transposes folded; attention "
                            "unfused (head dim D > 256)",
                "l2": "256 MiB written between timed steps (flush)"}

    def setup_e2e(self):
        t = self.torch
        self.hx = self.inputs[self.x_id].cpu().pin_memory()
        out = self.plan.tensor(self.out_id)
        self.hout = t.empty(out.shape, dtype=out.dtype).pin_memory()
        self.h2d = self.hx.numel() * 2
        self.d2h = self.hout.numel() * 2

    def step_e2e(self):
        self.inputs[self.x_id].copy_(self.hx, non_blocking=True)
        self.plan.run()
        self.hout.copy_(self.plan.tensor(self.out_id), non_blocking=True)
        self.torch.cuda.synchronize()

    def cpu_sample(self, lib, threads):
        return None


class RowWorkload(Workload):
    """x[65536x4096] fp32, rows over ranks."""
    R, Cc = 65536, 4096
    unit = "GB/s"
    bound = "hbm"
    dtype = "f32"

    KERNELS = {"rmsnorm_fwd": "norm_fwd_kernel", "layernorm_fwd": "norm_fwd_kernel",
               "rmsnorm_bwd": "norm_bwd_kernel", "layernorm_bwd": "norm_bwd_kernel",
               "reduce_max_fwd": "argmax_kernel", "reduce_max_bwd": "argmax_bwd_kernel",
               "softmax_fwd": "softmax_rows_kernel", "softmax_grad": "softmax_grad_kernel",
               "silu_grad": "silu_grad_kernel", "reduce_sum_rows": "row_sum_kernel",
               "reduce_sum_cols": "col_partial_kernel", "broadcast_rows": "broadcast_kernel"}

    def __init__(self, *a, op="rmsnorm_fwd"):
        super().__init__(*a)
        if op not in self.KERNELS:
            raise SystemExit(f"unknown workload {op}")
        self.op = op
        self.kernel = self.KERNELS[op]
        self.profile = f"{self.kernel}_{op}_config3"

    def setup(self):
        t = self.torch
        self.r0, self.r1 = split_rows(self.R, self.rank, self.world)
        self.m = self.r1 - self.r0
        g = t.Generator(device="cuda").manual_seed(3000 + self.r0)
        self.x = t.randn(self.m, self.Cc, device="cuda", generator=g)
        self.dy = t.randn(self.m, self.Cc, device="cuda", generator=g)
        self.g = 1 + 0.1 * t.randn(self.Cc, device="cuda", generator=g)
        self.bt = 0.1 * t.randn(self.Cc, device="cuda", generator=g)
        self.y = t.empty_like(self.x)
        self.dg = t.empty(self.Cc, device="cuda")
        self.db = t.empty(self.Cc, device="cuda")
        self.mx = t.empty(self.m, device="cuda")
        self.am = t.zeros(self.m, dtype=t.int32, device="cuda")
        self.dyr = self.dy[:, 0].contiguous()
        if self.op == "reduce_max_bwd":
            self.ctx.reduce_max_fwd(self.x, self.mx, self.am, self.m, self.Cc, self.Cc)

    def step(self):
        c, m, C_ = self.ctx, self.m, self.Cc
        if self.op == "rmsnorm_fwd":
            c.rmsnorm_fwd(self.x, self.y, self.g, self.bt, m, C_, C_, 1e-5); return 1
        if self.op == "layernorm_fwd":
            c.layernorm_fwd(self.x, self.y, self.g, self.bt, m, C_, C_, 1e-5); return 1
        if self.op == "rmsnorm_bwd":
            c.rmsnorm_bwd(self.x, self.g, self.dy, self.y, self.dg, self.db, m, C_, C_, 1e-5); return 2
        if self.op == "layernorm_bwd":
            c.layernorm_bwd(self.x, self.g, self.dy, self.y, self.dg, self.db, m, C_, C_, 1e-5); return 2
        if self.op == "reduce_max_fwd":
            c.reduce_max_fwd(self.x, self.mx, self.am, m, C_, C_); return 1
        if self.op == "reduce_max_bwd":
            c.reduce_max_bwd(self.am, self.dyr, self.y, m, C_, C_); return 1
        if self.op == "softmax_fwd":
            c.softmax_fwd(self.x, self.y, m, C_, C_); return 1
        if self.op == "softmax_grad":
            c.softmax_grad(self.x, self.dy, self.y, m, C_, C_); return 1
        if self.op == "silu_grad":
            c.silu_grad(self.x, self.dy, self.y, m * C_); return 1
        if self.op == "reduce_sum_rows":
            c.reduce_sum(self.x, self.mx, m, C_, C_, 1); return 1
        if self.op == "reduce_sum_cols":
            c.reduce_sum(self.x, self.dg, m, C_, C_, 0); return 2
        if self.op == "broadcast_rows":
            c.broadcast(self.dyr, self.y, m, C_, C_, 1); return 1
        raise ValueError(self.op)

    def bytes_for(self, rows):
        n = rows * self.Cc * 4
        return {"rmsnorm_fwd": 2 * n, "layernorm_fwd": 2 * n, "rmsnorm_bwd": 3 * n,
                "layernorm_bwd": 3 * n, "reduce_max_fwd": n + 8 * rows,
                "reduce_max_bwd": n + 8 * rows, "softmax_fwd": 2 * n, "softmax_grad": 3 * n,
                "silu_grad": 3 * n, "reduce_sum_rows": n + 4 * rows,
                "reduce_sum_cols": n + 4 * self.Cc, "broadcast_rows": n + 4 * rows}[self.op]

    def work_per_step(self):
        return float(self.bytes_for(self.m))

    def total_work_per_step(self):
        return float(self.bytes_for(self.R))

    def config(self):
        src = ("BASELINE configs[2], examples/norms" if "norm" in self.op or "max" in self.op
               else "autodiff graph op at the BASELINE configs[2] shape")
        return {"workload": f"{self.op} ({src})", "rows": self.R,
                "cols": self.Cc, "rows_per_gpu": self.m, "eps": 1e-5,
                "parallelism": f"rows over {self.world} GPU(s), no collective",
                "l2": "inputs (>= 1 GiB) larger than L2 and 256 MiB flush between steps"}

    def setup_e2e(self):
        self.hx = self.x.cpu().pin_memory()
        self.hy = self.torch.empty_like(self.hx).pin_memory()
        self.hg, self.hbt = self.g.cpu().pin_memory(), self.bt.cpu().pin_memory()
        self.h2d = (self.m * self.Cc + 2 * self.Cc) * 4
        self.d2h = self.m * self.Cc * 4

    def step_e2e(self):
        if self.op != "rmsnorm_fwd":
            raise NotImplementedError
        self.bwpp.rmsnorm_f32(self.hx, self.hy, self.hg, self.hbt, self.m, self.Cc, self.Cc, 1e-5)

    # the reference's own CPU function for this op (runtime/cpu/bwpp_cpu_ref.h), where
    # it has one: rmsnorm forward, softmax, and the reduce_max mask / grad pair (the
    # reference's form of the max and its routed gradient)
    REF_OPS = ("rmsnorm_fwd", "softmax_fwd", "reduce_max_fwd", "reduce_max_bwd")

    def cpu_sample(self, lib, threads):
        import ctypes as C

        import oracle as O
        if self.op not in self.REF_OPS:
            return None
        rows, cols = 4096, self.Cc
        rng = np.random.default_rng(3000)
        x = rng.standard_normal((rows, cols), dtype=np.float32)
        y = np.zeros_like(x)
        g = (1 + 0.1 * rng.standard_normal(cols)).astype(np.float32)
        dy = rng.standard_normal(rows).astype(np.float32)
        fp = C.POINTER(C.c_float)
        at = lambda a, r0: C.cast(C.c_void_p(a.ctypes.data + r0 * cols * 4), fp)
        if self.op == "reduce_max_bwd":
            lib.reduce_max_mask_f32(x.ctypes.data_as(fp), y.ctypes.data_as(fp), rows, cols, 1)

        def part(r0, r1):
            n = r1 - r0
            if self.op == "rmsnorm_fwd":
                lib.rmsnorm_f32(at(x, r0), at(y, r0), g.ctypes.data_as(fp), None, n, cols, cols, 1e-5)
            elif self.op == "softmax_fwd":
                lib.softmax_f32(at(x, r0), at(y, r0), n, cols, cols)
            elif self.op == "reduce_max_fwd":
                lib.reduce_max_mask_f32(at(x, r0), at(y, r0), n, cols, 1)
            else:  # gradient routed through the mask: dx = mask * dy[row]
                lib.reduce_max_grad_f32(at(y, r0), C.cast(C.c_void_p(dy.ctypes.data + r0 * 4), fp),
                                        at(x, r0), n, cols, 1)
        t0 = time.perf_counter()
        O.run_rows_threaded(part, rows, threads)
        dt = time.perf_counter() - t0
        fn = {"rmsnorm_fwd": "bwpp_cpu_rmsnorm_f32", "softmax_fwd": "bwpp_cpu_softmax_f32",
              "reduce_max_fwd": "bwpp_cpu_reduce_max_mask_f32 (axis 1)",
              "reduce_max_bwd": "bwpp_cpu_reduce_max_grad_f32 (axis 1, on its mask)"}[self.op]
        return (float(self.bytes_for(rows)), dt,
                f"{fn} on {rows} of 65536 rows, fp32, {threads} threads (credited with this "
                f"workload's algorithmic bytes per row)")


class TinyModelWorkload(Workload):
    """2-layer pre-RMSNorm decoder, d_model 2048, 16 x 128 heads
    (causal), SiLU-gated MLP 5632, seq 2048, batch 16 per GPU, MSE loss; forward +
    backward + NCCL gradient allreduce + SGD, data-parallel (weak scaling)."""
    L, D, H, F, B, S = 2, 2048, 16, 5632, 16, 2048
    kernel = "tiny_model step"
    profile = "tiny_model_step_config5"
    scaling = "weak"
    e2e_api = "bwpp_cuda_tiny_model_step with pinned host x / target, loss read back to host"

    def batch(self, r):
        """Rank r's inputs and targets (seeded per rank; any GPU regenerates them)."""
        t = self.torch
        g = t.Generator(device="cuda").manual_seed(5000 + r)
        x = t.randn(self.B * self.S, self.D, device="cuda", generator=g)
        return x, t.randn(self.B * self.S, self.D, device="cuda", generator=g)

    def setup(self):
        t = self.torch
        self.model = self.bwpp.TinyModel(self.ctx, self.L, self.D, self.H, self.F, self.B, self.S,
                                         1e-5, seed=1)
        self.x, self.tgt = self.batch(self.rank)
        self.loss = t.empty(1, device="cuda")
        self.comm = None
        if self.world > 1:
            import torch.distributed as dist
            self.comm = comm_from_process_group(self.bwpp.load(), self.rank, self.world,
                                                self.torch.cuda.current_device(), dist)

    def step(self):
        self.model.step(self.x, self.tgt, lr=1e-4, comm=self.comm, loss_out=self.loss)
        L = self.L
        # our kernel launches per step: forward 8 per layer (2 rmsnorm, 4 GEMMs,
        # attention, swiglu) + loss 2; backward 15 per layer (8 GEMMs, 2 rmsnorm
        # backward + 2 column sums, delta, dQ, dK/dV); SGD 1 (the allreduce is NCCL's)
        return L * 8 + 2 + L * 15 + 1

    def fwd_flops(self):
        T, D, F = self.B * self.S, self.D, self.F
        gemm = 2.0 * T * (3 * D * D + D * D + 2 * D * F + F * D)
        attn = 4.0 * self.B * self.H * 128 * self.S * (self.S + 1) / 2
        return self.L * (gemm + attn)

    def work_per_step(self):
        return 3.0 * self.fwd_flops()  # forward + backward ~ 3x forward

    def total_work_per_step(self):
        return self.world * self.work_per_step()

    def config(self):
        return {"workload": "tiny_model DP training step (BASELINE configs[4])", "layers": self.L,
                "d_model": self.D, "heads": self.H, "head_dim": 128, "ffn": self.F,
                "batch_per_gpu": self.B, "seq": self.S, "global_batch": self.B * self.world,
                "parallelism": f"data-parallel over {self.world} GPU(s), NCCL allreduce of "
                               "102.8M fp32 gradients",
                "flops": "3 x forward (GEMMs + causal attention)",
                "l2": "working set (GBs) far larger than L2"}

    def dp_check(self):
        """After the timed steps (every rank calls this; same collectives in the
        same order):
          replicas_bit_identical  every rank's fp32 parameters equal rank 0's bit
                                  for bit (NCCL broadcast + compare)
          allreduce_rel_err       one more step at lr = 0 gives the gradient summed
                                  over ranks; rank 0 regenerates every rank's batch,
                                  recomputes each gradient locally (no comm) and
                                  sums them: ||G - sum|| / ||sum|| (fp64)
          update_rel_err          the same for the SGD update -(lr / N) G"""
        t = self.torch
        n = self.model.count
        out = {"ranks": self.world}
        p = t.empty(n, device="cuda")
        self.model.get(p, None)
        if self.world > 1:
            import torch.distributed as dist
            ref = p.clone()
            dist.broadcast(ref, 0)
            same = t.tensor([1 if bool(t.equal(ref, p)) else 0], dtype=t.int32, device="cuda")
            dist.all_reduce(same, op=dist.ReduceOp.MIN)
            out["replicas_bit_identical"] = bool(same.item())
            del ref
        else:
            out["replicas_bit_identical"] = True
        self.model.step(self.x, self.tgt, lr=0.0, comm=self.comm)
        g = t.empty(n, device="cuda")
        self.model.get(None, g)
        if self.rank == 0:
            acc = t.zeros(n, dtype=t.float64, device="cuda")
            buf = t.empty(n, device="cuda")
            for r in range(self.world):
                xr, tr = self.batch(r)
                self.model.step(xr, tr, lr=0.0)
                self.model.get(None, buf)
                acc += buf.double()
                del xr, tr
            err = float(t.linalg.norm(g.double() - acc) / t.linalg.norm(acc))
            out["allreduce_rel_err"] = err
            out["update_rel_err"] = err  # the update is -(lr / N) times the summed gradient
            out["bound"] = "fp32 reassociation of the sum over ranks (NCCL order vs rank order)"
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()
        return out

    def setup_e2e(self):
        self.hx = self.x.cpu().pin_memory()
        self.ht = self.tgt.cpu().pin_memory()
        self.hloss = self.torch.empty(1).pin_memory()
        self.h2d = 2 * self.B * self.S * self.D * 4
        self.d2h = 4

    def step_e2e(self):
        self.model.step(self.hx, self.ht, lr=1e-4, comm=self.comm, loss_out=self.hloss)
        self.ctx.sync()

    def cpu_sample(self, lib, threads):
        return None


def make_workload(name, *a):
    if name == "gemm":
        return GemmWorkload(*a)
    if name == "tiny_model":
        return TinyModelWorkload(*a)
    if name == "gemm_f16":
        return GemmF16Workload(*a)
    if name == "plan_tiny_model":
        return PlanTinyModelWorkload(*a)
    if name in ("attention", "attention_causal"):
        return AttentionWorkload(*a, causal=name.endswith("causal"))
    if name in ("attention_f16", "attention_causal_f16"):
        return AttentionF16Workload(*a, causal="causal" in name)
    if name == "attention_bwd":
        return AttentionBwdWorkload(*a)
    return RowWorkload(*a, op=name)


# ---------------------------------------------------------------------------
# reference arm: the reference's own CPU code on the host cores
# ---------------------------------------------------------------------------

def reference_config(name, world):
    """The `config` our arm reports for this workload at this world size (rank 0's
    shard sizes), built without a GPU."""
    wl = make_workload(name, 0, world, None, None, None)
    if isinstance(wl, GemmWorkload):
        wl.r0, wl.r1 = split_rows(wl.M, 0, world)
        wl.m = wl.r1 - wl.r0
    elif isinstance(wl, AttentionWorkload):
        wl.h0, wl.h1 = split_rows(wl.B * wl.H, 0, world)
        wl.nh = wl.h1 - wl.h0
    elif isinstance(wl, AttentionBwdWorkload):
        wl.b0, wl.b1 = split_rows(wl.B, 0, world)
        wl.nb = wl.b1 - wl.b0
    elif isinstance(wl, RowWorkload):
        wl.r0, wl.r1 = split_rows(wl.R, 0, world)
        wl.m = wl.r1 - wl.r0
    try:
        return wl.config()
    except AttributeError:
        return {"workload": name}


def run_reference(args, world):
    import oracle as O
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    lib = O.ref_lib()
    kind = "reference"
    if lib is None:
        lib, kind = O.oracle_lib(), "port"
    threads = O.cpu_threads()
    wl = make_workload(args.workload, 0, 1, None, None, None)
    cfg = reference_config(args.workload, world)
    if wl.cpu_sample(lib, threads) is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          f"the reference has no CPU implementation of {args.workload}"}), flush=True)
        return
    for _ in range(args.warmup):
        wl.cpu_sample(lib, threads)
    work, secs = 0.0, 0.0
    sample = ""
    for _ in range(args.steps):
        w, dt, sample = wl.cpu_sample(lib, threads)
        work += w
        secs += dt
    value = wl.scale(work, secs)
    line = {"metric": METRIC, "value": value, "unit": wl.unit, "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * secs / max(args.steps, 1),
            "higher_is_better": True, "scaling": getattr(wl, "scaling", "strong"), "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded), fp32 copies of the benchmark inputs", "config": cfg,
            "cpu_baseline": {"value": value, "unit": wl.unit, "cores": threads, "kind": kind,
                             "sample": sample},
            "e2e": {"value": value, "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    # the same suite as our arm's "workloads": the reference's CPU code for each
    # config where it has one (median of 3 bounded samples)
    workloads = {}
    for name in suite_names(args.workloads, args.workload):
        sw = make_workload(name, 0, 1, None, None, None)
        cb = cpu_baseline_of(sw)
        if cb is None:
            workloads[name] = {"unavailable": f"the reference has no CPU implementation of {name}"}
        else:
            workloads[name] = {"value": cb["value"], "unit": cb["unit"], "cpu_baseline": cb,
                               "config": reference_config(name, world)}
    if workloads:
        line["workloads"] = workloads
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------

# The rest of BASELINE's configs, measured in the same default run (one
# workload at a time, each released before the next) and reported under
# "workloads" in the JSON line; the reference's bench/bench_cpu.c likewise
# covers matmul, softmax and rmsnorm in one run.
SUITE = ("attention", "attention_causal", "rmsnorm_fwd", "rmsnorm_bwd", "layernorm_fwd",
         "layernorm_bwd", "reduce_max_fwd", "reduce_max_bwd", "softmax_fwd", "tiny_model")


def suite_names(arg, primary):
    if arg in ("", "none"):
        return []
    names = SUITE if arg == "all" else tuple(n for n in arg.split(",") if n)
    return [n for n in names if n != primary]


def time_steps(wl, steps, warmup, torch, ctx, flush, barrier, dist, clocks=None):
    """W untimed steps, then K steps with CUDA events around each on the
    launching stream (an L2 flush before each); max over ranks of the sum."""
    stream = torch.cuda.current_stream()
    for _ in range(max(warmup, 0)):
        wl.step()
    ctx.sync()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
    launches = 0
    barrier()
    torch.cuda.synchronize()
    wall0 = time.perf_counter()
    for i in range(steps):
        flush.fill_(float(i))
        starts[i].record(stream)
        launches += wl.step()
        ends[i].record(stream)
        if clocks:
            clocks.poll()
    while not ends[-1].query():
        if clocks:
            clocks.poll()
        time.sleep(0.001)
    torch.cuda.synchronize()
    if clocks:
        clocks.poll(force=True)
    barrier()
    wall = time.perf_counter() - wall0
    ctx.sync()
    per_step_ms = [st.elapsed_time(en) for st, en in zip(starts, ends)]
    total_s = max_over_ranks(sum(per_step_ms) / 1e3, dist, "cuda")
    return total_s, sum(per_step_ms) / 1e3 / steps, launches, wall


def roofline_of(wl, my_launch_s):
    hbm, tflops, tflops_sus, src = peaks()
    achieved = wl.scale(wl.work_per_step(), my_launch_s)
    # a kernel timed alone is compared with the burst GEMM peak, a multi-kernel
    # training step (seconds of back-to-back work) with the sustained one
    peak = (tflops_sus if getattr(wl, "scaling", "") == "weak" else tflops) \
        if wl.unit == "TFLOP/s" else hbm
    # ncu dram bytes of one full-size (N = 1) launch, scaled to this rank's share
    traffic = profile_traffic(wl.profile)
    if traffic is not None:
        traffic = traffic * wl.work_per_step() / wl.total_work_per_step()
    r = {"bound": wl.bound, "achieved": achieved, "peak": peak, "unit": wl.unit,
         "frac": achieved / peak, "traffic": traffic,
         "peak_source": f"{src} (MEASURED_PEAKS.json)" if src == "measured" else "fallback",
         "kernel": wl.kernel}
    if getattr(wl, "scaling", "") == "weak":
        r["peak_kind"] = "bf16_tflops_sustained"
    return r


def cpu_baseline_of(wl, repeats=3):
    """The reference's own CPU code (oracle/_ref; the oracle port if absent) on
    a bounded sample of this workload: one warm-up call, then the median rate
    of `repeats` timed calls.  None where the reference has no CPU code."""
    import oracle as O
    lib, kind = O.ref_lib(), "reference"
    if lib is None:
        lib, kind = O.oracle_lib(), "port"
    threads = O.cpu_threads()
    if wl.cpu_sample(lib, threads) is None:
        return None
    rates, secs, sample = [], [], ""
    for _ in range(repeats):
        w, dt, sample = wl.cpu_sample(lib, threads)
        rates.append(wl.scale(w, dt))
        secs.append(dt)
    return {"value": float(np.median(rates)), "unit": wl.unit, "cores": threads, "kind": kind,
            "sample": sample, "repeats": repeats, "seconds": float(np.median(secs)),
            "spread": [float(min(rates)), float(max(rates))]}


def run_suite(names, args, rank, world, torch, bwpp, ctx, flush, barrier, dist):
    """Each workload in turn, released before the next.  A workload that fails
    is reported as {"error": ...} and ends the suite, so the headline line is
    still printed (every rank runs the same steps, so a failure that is not
    rank-local stops all ranks at the same point)."""
    out = {}
    for name in names:
        try:
            out[name] = run_workload(name, args, rank, world, torch, bwpp, ctx, flush, barrier, dist)
        except Exception as e:  # noqa: BLE001 - reported in the JSON line
            out[name] = {"error": f"{type(e).__name__}: {e}"[:400]}
            print(f"bench: workload {name} failed: {e}", file=sys.stderr, flush=True)
            break
    return out


def run_workload(name, args, rank, world, torch, bwpp, ctx, flush, barrier, dist):
    wl = make_workload(name, rank, world, torch, bwpp, ctx)
    if args.rows and isinstance(wl, RowWorkload):
        wl.R = args.rows
    wl.setup()
    total_s, my_s, launches, _ = time_steps(wl, args.steps, args.warmup, torch, ctx, flush,
                                            barrier, dist)
    entry = {"value": wl.scale(wl.total_work_per_step() * args.steps, total_s), "unit": wl.unit,
             "ms_per_step": 1e3 * total_s / args.steps, "scaling": getattr(wl, "scaling", "strong"),
             "dtype": wl.dtype, "gpu_launches": launches, "roofline": roofline_of(wl, my_s),
             "config": wl.config()}
    if hasattr(wl, "dp_check"):
        entry["dp_check"] = wl.dp_check()
    if rank == 0 and world == 1 and not args.no_cpu:
        entry["cpu_baseline"] = cpu_baseline_of(wl)
    if getattr(wl, "comm", None):
        torch.cuda.synchronize()
        bwpp.load().bwpp_cuda_comm_destroy(wl.comm)
        wl.comm = None
    if hasattr(wl, "model"):
        wl.model.close()
    del wl
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    barrier()
    return entry


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="gemm")
    ap.add_argument("--workloads", default=None,
                    help="extra workloads reported under 'workloads': all (default with the "
                         "gemm headline), none, or a comma list")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--rows", type=int, default=0,
                    help="row-workload rows (default 65536) or the GEMM's M (default 8192); "
                         "other values only for profiler captures")
    args = ap.parse_args()
    if args.workloads is None:
        args.workloads = "all" if args.workload == "gemm" else "none"
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.impl == "reference":
        run_reference(args, world)
        return

    import torch
    import torch.distributed as dist

    import bwpp
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    ctx = bwpp.Ctx(local)
    wl = make_workload(args.workload, rank, world, torch, bwpp, ctx)
    if args.rows and isinstance(wl, RowWorkload):
        wl.R = args.rows
    if args.rows and isinstance(wl, GemmWorkload):
        wl.M = args.rows  # e.g. the per-GPU share of an N-GPU run, for a profiler capture
    wl.setup()
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device="cuda")

    # ---- timed region: K steps, events around each step on the launch stream
    clocks = ClockSampler(local)
    total_s, my_launch_s, launches, wall = time_steps(wl, args.steps, args.warmup, torch, ctx,
                                                      flush, barrier, dist, clocks)
    value = wl.scale(wl.total_work_per_step() * args.steps, total_s)
    ms_per_step = 1e3 * total_s / args.steps

    # ---- roofline of the dominant kernel (this rank's launches)
    roofline = roofline_of(wl, my_launch_s)

    # ---- e2e through the C ABI mirror with host buffers
    e2e = None
    if not args.no_e2e:
        try:
            wl.setup_e2e()
            for _ in range(max(1, min(args.warmup, 2))):
                wl.step_e2e()
            n_e2e = max(3, min(args.steps, 10))
            barrier()
            t0 = time.perf_counter()
            for _ in range(n_e2e):
                wl.step_e2e()
            dt = max_over_ranks(time.perf_counter() - t0, dist, "cuda")
            e2e = {"value": wl.scale(wl.total_work_per_step() * n_e2e, dt), "unit": wl.unit,
                   "h2d_bytes_per_step": int(wl.h2d), "d2h_bytes_per_step": int(wl.d2h), "steps": n_e2e,
                   "api": getattr(wl, "e2e_api", "bwpp_cuda_*_f32 CPU-signature mirror, pinned host buffers")}
        except NotImplementedError:
            e2e = None

    # ---- CPU baseline: the reference's own code on this host (rank 0, N = 1)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline_of(wl)

    dp = wl.dp_check() if hasattr(wl, "dp_check") else None
    if getattr(wl, "comm", None):
        torch.cuda.synchronize()
        bwpp.load().bwpp_cuda_comm_destroy(wl.comm)
        wl.comm = None
    line = {"metric": METRIC, "value": value, "unit": wl.unit, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": getattr(wl, "scaling", "strong"), "vs_baseline": None, "dtype": wl.dtype,
            "data": "synthetic (seeded torch generators), shapes and distributions of the BASELINE config",
            "config": wl.config(), "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e,
            "gpu_launches": launches, "clocks": clocks.summary(), "wall_s_timed_region": wall}
    if dp is not None:
        line["dp_check"] = dp

    # ---- the other BASELINE configs, each measured the same way
    names = suite_names(args.workloads, args.workload)
    if names:
        if hasattr(wl, "model"):
            wl.model.close()
        del wl
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        line["workloads"] = run_suite(names, args, rank, world, torch, bwpp, ctx, flush, barrier, dist)
    if world > 1:
        dist.barrier()
    if rank == 0:
        print(json.dumps(line), flush=True)
    ctx.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
