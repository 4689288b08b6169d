"""bench.py's reference arm, on CPU: it reports the CUDA arm's config for the
same workload and world size, and prints an `unavailable` line (exit 0) for a
workload the reference has no CPU code for."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


@pytest.mark.parametrize("name,world,key,value", [
    ("gemm", 8, "rows_per_gpu", 1024),
    ("gemm", 1, "rows_per_gpu", 8192),
    ("attention_causal", 4, "heads_per_gpu", 64),
    ("rmsnorm_bwd", 2, "rows_per_gpu", 32768),
    ("attention_bwd", 4, "batch_per_gpu", 4),
    ("tiny_model", 8, "global_batch", 128),
])
def test_reference_config_matches_the_cuda_arm(name, world, key, value):
    cfg = bench.reference_config(name, world)
    assert cfg[key] == value
    assert cfg["workload"] != name  # the descriptive config, not the bare name


def _reference_line(workload):
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--workload", workload, "--steps", "1", "--warmup", "0"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    return json.loads(out.stdout.strip().splitlines()[-1])


def test_reference_arm_without_cpu_code_prints_unavailable():
    d = _reference_line("tiny_model")
    assert d["impl"] == "reference" and "no CPU implementation" in d["unavailable"]


def test_reference_arm_row_op_uses_the_reference_function():
    d = _reference_line("softmax_fwd")
    assert d["impl"] == "reference" and d["value"] > 0 and d["unit"] == "GB/s"
    assert "bwpp_cpu_softmax_f32" in d["cpu_baseline"]["sample"]
    assert d["config"]["rows_per_gpu"] == 65536
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


@pytest.mark.parametrize("name", ["gemm_tc_kernel_config2", "attention_tc_kernel_config4",
                                  "attention_bwd_tiny_model", "norm_fwd_kernel_rmsnorm_fwd_config3",
                                  "softmax_rows_kernel_softmax_fwd_config3"])
def test_profile_traffic_is_recorded(name):
    """The roofline's `traffic` comes from the committed ncu summary of the kernel."""
    traffic = bench.profile_traffic(name)
    assert traffic is not None and traffic > 1e8


def test_default_run_covers_every_baseline_config():
    """The headline GEMM run also measures attention (both masks), the norms,
    reduce_max, softmax and the tiny_model DP step; other workloads run alone."""
    names = bench.suite_names("all", "gemm")
    for n in ("attention", "attention_causal", "rmsnorm_fwd", "rmsnorm_bwd", "layernorm_fwd",
              "layernorm_bwd", "reduce_max_fwd", "reduce_max_bwd", "softmax_fwd", "tiny_model"):
        assert n in names
    assert "gemm" not in names
    assert bench.suite_names("none", "gemm") == []
    assert bench.suite_names("attention,tiny_model", "tiny_model") == ["attention"]


def test_reference_arm_default_reports_the_suite():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "0"],
                         capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads(out.stdout.strip().splitlines()[-1])
    w = d["workloads"]
    assert w["rmsnorm_fwd"]["unit"] == "GB/s" and w["rmsnorm_fwd"]["value"] > 0
    assert w["attention_causal"]["unit"] == "TFLOP/s"
    assert w["rmsnorm_fwd"]["cpu_baseline"]["repeats"] == 3
    assert "unavailable" in w["tiny_model"] and "unavailable" in w["layernorm_bwd"]


def test_a_failing_workload_is_reported_and_ends_the_suite(monkeypatch):
    """A workload that raises is reported as {"error": ...}; the suite stops
    there, so the headline JSON line is still printed."""
    ran = []

    def fake(name, *a, **k):
        ran.append(name)
        if name == "rmsnorm_fwd":
            raise RuntimeError("boom")
        return {"value": 1.0}

    monkeypatch.setattr(bench, "run_workload", fake)
    out = bench.run_suite(["attention", "rmsnorm_fwd", "softmax_fwd"], None, 0, 1, None, None, None,
                          None, None, None)
    assert ran == ["attention", "rmsnorm_fwd"]
    assert out["attention"] == {"value": 1.0}
    assert out["rmsnorm_fwd"]["error"].startswith("RuntimeError: boom")
    assert "softmax_fwd" not in out
