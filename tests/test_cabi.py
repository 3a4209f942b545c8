"""The C-ABI library loads and exports every entry point include/sbq.h declares (no GPU needed)."""

import ctypes
import re
from pathlib import Path

import pytest

from conftest import ROOT


def declared_functions():
    text = (ROOT / "include" / "sbq.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"^\s*SBQ_API\s+(?:const\s+)?\w+\**\s+\**(sbq_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_entry_points():
    names = declared_functions()
    assert "sbq_gemv_w8" in names and "sbq_linear_dyn" in names and len(names) >= 16


def test_library_exports_every_declared_symbol(sbq):
    lib = sbq._lib.load()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_header(sbq):
    assert set(declared_functions()) == set(sbq._lib.SIGNATURES)


def test_host_side_calls_without_gpu(sbq):
    lib = sbq._lib.load()
    assert lib.sbq_version() >= 10000
    assert lib.sbq_packed_bytes(16, 64) == 1024
    assert lib.sbq_packed_bytes(17, 65) == 4096
    assert lib.sbq_packed_bytes(0, 64) == 0
    assert lib.sbq_status_string(0) == b"SBQ_OK"


def test_argument_errors_raise_before_launch(sbq):
    L = sbq._lib
    # a null weight pointer is rejected on the host with ValueError (no device touched)
    with pytest.raises(ValueError, match="SBQ_ERR_INVALID_ARGUMENT"):
        L.call("sbq_gemv_w8", ctypes.c_void_p(16), L.F16, 64, None, None, None, 1, 16, 64, ctypes.c_void_p(16),
               L.F32, 16, None)
    with pytest.raises(ValueError, match="SBQ_ERR_UNSUPPORTED"):
        L.call("sbq_gemv_w8", ctypes.c_void_p(256), 7, 64, ctypes.c_void_p(256), ctypes.c_void_p(256), None, 1, 16,
               64, ctypes.c_void_p(256), L.F32, 16, None)
    with pytest.raises(ValueError, match="SBQ_ERR_ALIGNMENT"):
        L.call("sbq_gemv_w8", ctypes.c_void_p(8), L.F16, 64, ctypes.c_void_p(256), ctypes.c_void_p(256), None, 1, 16,
               64, ctypes.c_void_p(256), L.F32, 16, None)
    with pytest.raises(ValueError, match="multiple of 16"):
        L.call("sbq_gemv_w8", ctypes.c_void_p(256), L.F16, 72, ctypes.c_void_p(256), ctypes.c_void_p(256), None, 1,
               16, 72, ctypes.c_void_p(256), L.F32, 16, None)


def test_make_linear_unknown_format(sbq):
    import torch
    with pytest.raises(ValueError, match="unknown weight format"):
        sbq.make_linear("int4", torch.zeros(4, 4))


def test_package_surface(sbq):
    # the drop-in names of spikingbrain_cpu/quant.py plus the stack and MLP modules
    for name in ("FORMATS", "quantize_per_channel", "Int8Linear", "DynamicInt8Linear", "FP16Linear", "BF16Linear",
                 "FloatLinear", "make_linear", "FusedGatedMLP", "fuse_gated_mlp", "stack", "workloads"):
        assert hasattr(sbq, name), name
    assert sbq.FORMATS == ("float32", "bfloat16", "float16", "int8", "int8-dyn")
    assert hasattr(sbq.stack, "ProjectionStack") and hasattr(sbq.stack, "CapturedStack")


def test_peer_group_arguments_rejected_on_the_host(sbq):
    """Argument checks of the sharded launch run before any CUDA call (no GPU needed)."""
    import ctypes

    L = sbq._lib
    lib = L.load()
    job = L.GemvJob(16, 64, 256, 256, None, None, None, 16, 64, 512, L.F32, 16)
    jobs = (L.GemvJob * 1)(job)
    assert lib.sbq_gemv_w8_group_peer(jobs, 1, L.F16, 1, None, None) == L.ERR_INVALID_ARGUMENT
    pg = L.PeerGroup()
    pg.nranks = 0
    assert lib.sbq_gemv_w8_group_peer(jobs, 1, L.F16, 1, ctypes.byref(pg), None) == L.ERR_INVALID_ARGUMENT
    pg.nranks = 9
    assert lib.sbq_gemv_w8_group_peer(jobs, 1, L.F16, 1, ctypes.byref(pg), None) == L.ERR_INVALID_ARGUMENT
    pg.nranks = 1
    pg.wait_count = 4096
    pg.wait_state = None
    assert lib.sbq_gemv_w8_group_peer(jobs, 1, L.F16, 1, ctypes.byref(pg), None) == L.ERR_INVALID_ARGUMENT
    assert lib.sbq_peer_wait(None, None, 1, 0, None) == L.ERR_INVALID_ARGUMENT
    assert lib.sbq_peer_wait(4100, 4096, 1, 0, None) == L.ERR_ALIGNMENT


def test_ready_job_counts_rejected_on_the_host(sbq):
    """sbq_gemv_w8_group_ready / _peer_ready check n_ready (0..njobs) before any CUDA call."""
    import ctypes

    L = sbq._lib
    lib = L.load()
    job = L.GemvJob(16, 64, 256, 256, None, None, None, 16, 64, 512, L.F32, 16)
    jobs = (L.GemvJob * 2)(job, job)
    for n_ready in (-1, 3):
        assert lib.sbq_gemv_w8_group_ready(jobs, 2, n_ready, L.F16, 1, None) == L.ERR_INVALID_ARGUMENT
        assert b"n_ready" in lib.sbq_last_error()
        pg = L.PeerGroup()
        pg.nranks = 1
        assert lib.sbq_gemv_w8_group_peer_ready(jobs, 2, n_ready, L.F16, 1, ctypes.byref(pg), None) == \
            L.ERR_INVALID_ARGUMENT
    assert lib.sbq_gemv_w8_group_peer_ready(jobs, 2, 1, L.F16, 1, None, None) == L.ERR_INVALID_ARGUMENT
