"""The no-allocation int8-dyn entry point against the workspace one.

Some callers of this library cannot call cudaMalloc (a runtime that owns all device memory through
its own pool, a C / FFI host that only holds raw pointers, a decode loop that must not synchronise
the device).  ``sbq_linear_dyn_noalloc`` serves them with a fixed scratch array inside the library.
These tests call it through the C ABI and require the same output as ``sbq_linear_dyn`` with a
caller workspace, bit for bit (the int8-dyn parity bar), on two calls in a row, so whatever the
first call leaves in the shared array cannot leak into the second.  This file is named to be
collected last.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import quant_ref as R

pytestmark = pytest.mark.gpu

_DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}  # SBQ_F32, SBQ_F16, SBQ_BF16


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _noalloc(lib, mod, x, y, mode_code):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    m, k = x.shape
    return lib.sbq_linear_dyn_noalloc(_p(x), _DTYPE_CODE[x.dtype], x.stride(0), mode_code,
                                      _p(mod.packed), _p(mod.rowsum), _p(mod.scale), _p(mod.bias), m,
                                      mod.out_features, k, _p(y), y.stride(0), stream)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("mode", ["per_tensor", "per_token"])
def test_noalloc_matches_workspace_entry_point_twice(sbq, mode, dtype):
    lib = sbq._lib.load()
    m, n, k = 96, 384, 1024
    w = sbq.workloads.float_weight(n, k, seed=71)
    bias = torch.randn(n)
    mod = sbq.DynamicInt8Linear(w, bias, mode=mode)
    code = sbq._lib.ACT_PER_TENSOR if mode == "per_tensor" else sbq._lib.ACT_PER_TOKEN
    for call, scale in enumerate((1.0, 7.5)):
        x = (sbq.workloads.activation(m, k, seed=72 + call, dtype=torch.float32) * scale).to(dtype).cuda()
        want = mod(x)  # sbq_linear_dyn with a caller-provided workspace
        y = torch.full((m, n), float("nan"), device="cuda")
        assert _noalloc(lib, mod, x, y, code) == 0, lib.sbq_last_error().decode()
        torch.cuda.synchronize()
        assert torch.equal(y, want), "call %d differs from sbq_linear_dyn" % call
    assert lib.sbq_check_device_error() == 0


def test_noalloc_matches_reference_oracle(sbq):
    lib = sbq._lib.load()
    m, n, k = 33, 200, 512
    w = sbq.workloads.float_weight(n, k, seed=74)
    mod = sbq.DynamicInt8Linear(w, None)
    x = sbq.workloads.activation(m, k, seed=75, dtype=torch.float32)
    y = torch.empty(m, n, device="cuda")
    assert _noalloc(lib, mod, x.cuda(), y, sbq._lib.ACT_PER_TENSOR) == 0
    q, s = R.quantize_per_channel(w.numpy())
    want = R.dyn_linear(x.numpy(), q, s)[0]
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_noalloc_rejects_sizes_beyond_its_array(sbq):
    lib = sbq._lib.load()
    m, n, k = 1021, 16, 4096  # needs 4 MiB + 256 bytes of scratch
    assert lib.sbq_dyn_workspace_bytes(m, k, 0) > (4 << 20)
    mod = sbq.DynamicInt8Linear(sbq.workloads.float_weight(n, k, seed=76), None)
    x = torch.zeros(m, k, device="cuda")
    y = torch.empty(m, n, device="cuda")
    status = _noalloc(lib, mod, x, y, sbq._lib.ACT_PER_TENSOR)
    assert status == sbq._lib.ERR_WORKSPACE
    assert "scratch" in lib.sbq_last_error().decode()
