"""C ABI surface of lib/libbwpp_cuda.so, checked without a GPU."""
import ctypes as C
import subprocess

import pytest

import bwpp


def test_library_exports_every_header_symbol():
    lib = bwpp.load()
    declared = bwpp.header_symbols()
    assert len(declared) >= 30
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    # the Python layer binds exactly what the header declares
    assert sorted(bwpp._SIGS) == declared


def test_only_api_symbols_are_exported():
    out = subprocess.run(["nm", "-D", "--defined-only", bwpp.LIB_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    ours = {s for s in exported if s.startswith("bwpp")}
    assert ours == set(bwpp.header_symbols())


def test_param_struct_layouts_match_metal_abi():
    # runtime/metal/dispatch_stub.h:9-40: all-uint32 structs (+ one float)
    assert C.sizeof(bwpp.MatmulParams) == 24
    assert C.sizeof(bwpp.SoftmaxParams) == 12
    assert C.sizeof(bwpp.RmsnormParams) == 16
    assert C.sizeof(bwpp.AttentionParams) == 32
    # runtime/core/arena.h:6-10
    assert C.sizeof(bwpp.Arena) == 24


def test_status_strings():
    for code in range(7):
        assert bwpp.status_string(code)
    assert bwpp.status_string(bwpp.ERR_TIMEOUT) == "device wait timed out"


def test_no_gpu_behaviour_is_an_error_not_a_crash():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    lib = bwpp.load()
    assert lib.bwpp_cuda_device_count() == 0
    h = C.c_void_p()
    assert lib.bwpp_cuda_ctx_create(C.byref(h), 0, None) == bwpp.ERR_ARG
    assert lib.bwpp_cuda_sync(None) == bwpp.ERR_ARG
    arena = bwpp.Arena()
    assert lib.bwpp_cuda_arena_init(C.byref(arena), 1 << 20, 0) == 0
    assert lib.bwpp_cuda_arena_alloc(C.byref(arena), 16, 16) is None
