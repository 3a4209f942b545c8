"""GPU parity of the W8A16 prefill GEMM (tcgen05 kind::f16, int8 tiles dequantised in shared memory).

Reference: Int8Linear.forward (spikingbrain_cpu/quant.py:41-53) at prefill shapes.  Tolerance:
relative L2 1e-3 (fp16 output rounding alone contributes ~3e-4), against the float64 oracle.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import quant_ref as R

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3


def _gemm(sbq, mod, x, y):
    L = sbq._lib
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731
    L.call("sbq_gemm_w8a16", p(x), L.F16, x.stride(0), p(mod.packed), p(mod.scale), p(mod.bias), x.shape[0],
           mod.out_features, x.shape[1], p(y), L.F32 if y.dtype == torch.float32 else L.F16, y.stride(0),
           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return y


def test_config2_prefill_gemm(sbq):
    cfg = sbq.workloads.CONFIGS[2]
    m, k, n = cfg["m"], cfg["k"], cfg["n"]
    w = sbq.workloads.float_weight(n, k, seed=50)
    x = sbq.workloads.activation(m, k, seed=51)
    q, s = R.quantize_per_channel(w.numpy())
    mod = sbq.Int8Linear(w, None)
    mod.out_dtype = torch.float16  # the configuration's fp16 output
    y = mod(x.cuda())
    assert y.dtype == torch.float16
    rows = np.array([0, 1, 127, 128, 1000, 1023, 1024, 2046, 2047])
    want = R.int8_linear(x.float().numpy()[rows], q, s)
    assert R.rel_l2(y.float().cpu().numpy()[rows], want) < REL_L2
    assert sbq._lib.load().sbq_check_device_error() == 0


@pytest.mark.parametrize("m,n,k", [(65, 130, 320), (128, 256, 64), (129, 300, 4096), (300, 1000, 128),
                                   (257, 4, 256), (200, 4096, 2560), (512, 12288, 4096), (1000, 512, 12288)])
@pytest.mark.parametrize("out", [torch.float32, torch.float16])
def test_gemm_shapes(sbq, m, n, k, out):
    w = sbq.workloads.float_weight(n, k, seed=m + k)
    x = sbq.workloads.activation(m, k, seed=n)
    b = torch.randn(n) if n % 2 else None
    q, s = R.quantize_per_channel(w.numpy())
    mod = sbq.Int8Linear(w, b)
    y = _gemm(sbq, mod, x.cuda(), torch.empty(m, n, dtype=out, device="cuda"))
    rows = np.unique(np.linspace(0, m - 1, 17).astype(int))
    want = R.int8_linear(x.float().numpy()[rows], q, s, None if b is None else b.numpy())
    assert R.rel_l2(y.float().cpu().numpy()[rows], want) < REL_L2


@pytest.mark.parametrize("m", [1, 17, 64])
def test_gemm_small_m_direct(sbq, m):
    n, k = 384, 512
    w = sbq.workloads.float_weight(n, k, seed=m)
    x = sbq.workloads.activation(m, k, seed=m + 1)
    q, s = R.quantize_per_channel(w.numpy())
    mod = sbq.Int8Linear(w, None)
    y = _gemm(sbq, mod, x.cuda(), torch.empty(m, n, device="cuda"))
    assert R.rel_l2(y.cpu().numpy(), R.int8_linear(x.float().numpy(), q, s)) < REL_L2


def test_linear_dispatch_gemm_matches_gemv(sbq):
    # the same layer through the GEMM (m > 64) and through the GEMV in 16-row passes agree
    n, k, m = 256, 1024, 96
    w = sbq.workloads.float_weight(n, k, seed=60)
    x = sbq.workloads.activation(m, k, seed=61).cuda()
    mod = sbq.Int8Linear(w, None)
    y_gemm = mod(x)
    L = sbq._lib
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    y_gemv = torch.empty(m, n, device="cuda")
    L.call("sbq_gemv_w8", p(x), L.F16, k, p(mod.packed), p(mod.scale), None, m, n, k, p(y_gemv), L.F32, n,
           ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert R.rel_l2(y_gemm.cpu().numpy(), y_gemv.cpu().numpy()) < 1e-5


def test_prefill_mlp_through_gemm(sbq):
    n, k, m = 1024, 512, 200
    ws = [sbq.workloads.float_weight(*sh, seed=70 + i) for i, sh in enumerate([(n, k), (n, k), (k, n)])]
    mlp = sbq.FusedGatedMLP(*(sbq.Int8Linear(w, None) for w in ws))
    x = sbq.workloads.activation(m, k, seed=73)
    y = mlp(x.cuda())
    o = [R.quantize_per_channel(w.numpy()) for w in ws]
    want = R.gated_mlp(x.float().numpy(), o[0], o[1], o[2], h_dtype=np.float16)
    assert R.rel_l2(y.cpu().numpy(), want) < REL_L2


@pytest.mark.parametrize("m,n,k", [(64, 256, 4096), (100, 4096, 4096), (33, 1000, 12288), (17, 130, 320),
                                   (128, 12288, 4096), (50, 4096, 12288)])
@pytest.mark.parametrize("out", [torch.float32, torch.float16])
def test_gemm_small_batch_split_k(sbq, m, n, k, out):
    # up to 128 rows: 64-token tiles; few tiles: the K range is split over a thread-block cluster
    # whose CTAs add their partial tiles through distributed shared memory in part order
    w = sbq.workloads.float_weight(n, k, seed=m * 7 + n)
    x = sbq.workloads.activation(m, k, seed=k + 3)
    b = torch.randn(n) if n % 3 else None
    q, s = R.quantize_per_channel(w.numpy())
    mod = sbq.Int8Linear(w, b)
    y1 = _gemm(sbq, mod, x.cuda(), torch.empty(m, n, dtype=out, device="cuda"))
    y2 = _gemm(sbq, mod, x.cuda(), torch.empty(m, n, dtype=out, device="cuda"))
    assert torch.equal(y1, y2)
    want = R.int8_linear(x.float().numpy(), q, s, None if b is None else b.numpy())
    assert R.rel_l2(y1.float().cpu().numpy(), want) < REL_L2
    assert sbq._lib.load().sbq_check_device_error() == 0


@pytest.mark.parametrize("m", [40, 64, 300])
@pytest.mark.parametrize("h_dtype", [torch.float16, torch.float32])
def test_gated_gemm_gateup(sbq, m, h_dtype):
    # above 32 rows the gate/up pair runs as two GEMMs: the gate projection into h, then the up
    # projection whose epilogue replaces it by silu(gate) * up (the gate is rounded to h's dtype)
    n, k = 1536, 1024
    wg = sbq.workloads.float_weight(n, k, seed=m + 1)
    wu = sbq.workloads.float_weight(n, k, seed=m + 2)
    wd = sbq.workloads.float_weight(k, n, seed=m + 3)
    mlp = sbq.FusedGatedMLP(*(sbq.Int8Linear(w, None) for w in (wg, wu, wd)), h_dtype=h_dtype)
    x = sbq.workloads.activation(m, k, seed=m + 4)
    h = mlp.gateup_into(x.cuda(), torch.empty(m, n, dtype=h_dtype, device="cuda"))
    g, u = (R.int8_linear(x.float().numpy(), *R.quantize_per_channel(w.numpy())) for w in (wg, wu))
    if h_dtype == torch.float16:
        g = g.astype(np.float16).astype(np.float64)
    want = g / (1.0 + np.exp(-g)) * u
    assert R.rel_l2(h.float().cpu().numpy(), want) < REL_L2
