"""Shared test setup.

`gpu` tests run the CUDA library on a B200 and compare it with the CPU oracle
(oracle/); everything else runs on CPU (oracle pinning, ABI surface, host
logic, gloo multi-rank logic).
"""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for sub in ("", "oracle", "bluewolf-plus-plus_b200"):
    p = os.path.join(ROOT, sub)
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 GPU (sm_100a)")


def rel_fro(a, b):
    """||a - b||_F / ||b||_F in float64."""
    import numpy as np
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


@pytest.fixture(scope="session")
def ctx():
    import torch
    import bwpp
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    c = bwpp.Ctx(0)
    yield c
    c.sync()
    c.close()


def dev(a):
    """numpy -> CUDA tensor (uint16 bf16 bits travel as int16)."""
    import numpy as np
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        return torch.from_numpy(a.view(np.int16)).cuda()
    if a.dtype == np.uint32:
        return torch.from_numpy(a.view(np.int32)).cuda()
    return torch.from_numpy(a).cuda()


def host(t, dtype=None):
    import numpy as np
    a = t.detach().cpu().numpy()
    if dtype is not None:
        a = a.view(dtype)
    return a


def empty_f32(*shape):
    import torch
    return torch.full(shape, float("nan"), dtype=torch.float32, device="cuda")
