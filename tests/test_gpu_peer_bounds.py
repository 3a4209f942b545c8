"""Bounded waits of the sharded decode path, made to run out on purpose (no GPU fault involved).

A wait whose signal nothing ever increments stops after its limit (50 ms here), records
SBQ_ERR_TIMEOUT for sbq_check_device_error and lets the kernel finish; the context stays usable and
a later wait that is satisfied passes.  One GPU, one rank.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import quant_ref as R

pytestmark = pytest.mark.gpu

LIMIT_NS = 50_000_000


def _arena(L, nbytes):
    ptr = ctypes.c_void_p()
    L.call("sbq_peer_alloc", nbytes, ctypes.byref(ptr))
    return ptr.value


def test_peer_wait_kernel_times_out_and_reports(sbq):
    L = sbq._lib
    lib = L.load()
    assert lib.sbq_check_device_error() == 0
    base = _arena(L, 16384)
    try:
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        L.call("sbq_peer_wait", ctypes.c_void_p(base), ctypes.c_void_p(base + 8192), 1, LIMIT_NS, stream)
        torch.cuda.synchronize()
        assert lib.sbq_check_device_error() == L.ERR_TIMEOUT
        assert lib.sbq_check_device_error() == 0  # reading the error clears it
        # the device still works
        w = sbq.workloads.float_weight(64, 256, seed=1)
        x = sbq.workloads.activation(1, 256, seed=2)
        q, s = R.quantize_per_channel(w.numpy())
        y = sbq.Int8Linear(w, None)(x.cuda())
        assert R.rel_l2(y.cpu().numpy(), R.int8_linear(x.float().numpy(), q, s)) < 1e-3
    finally:
        L.call("sbq_peer_free", ctypes.c_void_p(base))


def test_peer_group_wait_times_out_then_passes_when_signalled(sbq):
    L = sbq._lib
    lib = L.load()
    lib.sbq_check_device_error()  # start from a clear error word
    n, k = 256, 512
    mod = sbq.Int8Linear(sbq.workloads.float_weight(n, k, seed=3), None)
    x = sbq.workloads.activation(1, k, seed=4).cuda()
    want = mod(x)
    base = _arena(L, 65536)
    sig_a, sig_b, done, st1, st2 = base, base + 4096, base + 8192, base + 8448, base + 8704
    try:
        stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for wait_on, state, expect_timeout in ((sig_a, st1, True), (sig_b, st2, False)):
            y = torch.zeros(1, n, device="cuda")
            job = mod.gemv_job(x, y)
            pg = L.PeerGroup()
            pg.nranks = 1
            pg.y[0][0] = y.data_ptr()
            pg.signal[0] = sig_b  # each launch signals sig_b: the second launch's wait is satisfied
            pg.done = done
            pg.wait_count = wait_on
            pg.wait_state = state
            pg.wait_expected = 1
            pg.wait_limit_ns = LIMIT_NS
            L.call("sbq_gemv_w8_group_peer", (L.GemvJob * 1)(job), 1, L.F16, 1, ctypes.byref(pg), stream)
            torch.cuda.synchronize()
            status = lib.sbq_check_device_error()
            assert status == (L.ERR_TIMEOUT if expect_timeout else 0)
            # the kernel carried on after the wait: its own inputs were valid, so is its output
            assert torch.equal(y, want)
    finally:
        L.call("sbq_peer_free", ctypes.c_void_p(base))
