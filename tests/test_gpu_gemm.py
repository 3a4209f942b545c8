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
                                   (257, 4, 256), (200, 4096, 2560), (512, 12288, 4096), (1000, 512, 12288),
                                   (300, 640, 320), (260, 136, 336)])
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


@pytest.mark.parametrize("m", [17, 32, 40, 64, 300])
@pytest.mark.parametrize("h_dtype", [torch.float16, torch.float32])
def test_gated_gemm_gateup(sbq, m, h_dtype):
    # above 16 rows the gate/up pair runs as two GEMMs: the gate projection into h, then the up
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


# ---- fp32 and bf16 activations on the tensor-memory GEMM ------------------------------------------
# The reference's model feeds fp32 activations to every projection, in prefill chunks of up to 512
# tokens (model.py:439-441, quant.py:47).  Above 16 rows the drop-in splits fp32 x into bf16 high and
# low parts (sbq_linear_w8_ws) and the GEMM runs one MMA per part; bf16 x runs on the GEMM directly.
F32_REL_L2 = 2e-5  # the fp32 GEMV's bar: the split keeps ~17 significant bits of x


def _ws_bytes(sbq, m, k, dtype):
    return int(sbq._lib.load().sbq_linear_w8_workspace_bytes(m, k, {torch.float32: 0, torch.float16: 1,
                                                                       torch.bfloat16: 2}[dtype]))


@pytest.mark.parametrize("m,n,k", [(33, 4096, 2560), (100, 1024, 2560), (512, 4096, 2560), (512, 2560, 9728),
                                   (300, 130, 320), (2048, 512, 4096)])
def test_f32_prefill_on_tensor_cores(sbq, m, n, k):
    assert _ws_bytes(sbq, m, k, torch.float32) == 4 * m * k + (0 if (2 * m * k) % 256 == 0 else 2 * (256 - (2 * m * k) % 256))
    w = sbq.workloads.float_weight(n, k, seed=m + 3 * n)
    b = torch.randn(n) if m % 2 else None
    x = sbq.workloads.activation(m, k, seed=k + 5, dtype=torch.float32) * 3.0
    q, s = R.quantize_per_channel(w.numpy())
    y = sbq.Int8Linear(w, b)(x.cuda())
    rows = np.unique(np.linspace(0, m - 1, 48).astype(int))
    want = R.int8_linear(x.numpy()[rows], q, s, None if b is None else b.numpy())
    assert R.rel_l2(y.cpu().numpy()[rows], want) < F32_REL_L2


def test_config2_with_fp32_activations(sbq):
    # configuration 2's shape with the reference's own activation type: every 256-token tile sampled
    m, k, n = 2048, 4096, 12288
    w = sbq.workloads.float_weight(n, k, seed=50)
    x = sbq.workloads.activation(m, k, seed=51, dtype=torch.float32)
    q, s = R.quantize_per_channel(w.numpy())
    y = sbq.Int8Linear(w, None)(x.cuda()).cpu().numpy()
    rows = np.array(sorted({r for t in range(0, m, 256) for r in (t, t + 129, t + 255)}))
    assert R.rel_l2(y[rows], R.int8_linear(x.numpy()[rows], q, s)) < F32_REL_L2
    col_want = (x.numpy().astype(np.float64).sum(0) @ q.T.astype(np.float64)) * s
    assert R.rel_l2(y.astype(np.float64).sum(0), col_want) < F32_REL_L2


@pytest.mark.parametrize("m", [40, 128, 300])
@pytest.mark.parametrize("out", [torch.float32, torch.float16])
def test_bf16_activations_on_tensor_cores(sbq, m, out):
    n, k = 1000, 1024
    w = sbq.workloads.float_weight(n, k, seed=m + 9)
    x = sbq.workloads.activation(m, k, seed=m + 10, dtype=torch.bfloat16)
    assert _ws_bytes(sbq, m, k, torch.bfloat16) == 0
    q, s = R.quantize_per_channel(w.numpy())
    mod = sbq.Int8Linear(w, None)
    mod.out_dtype = out
    y = mod(x.cuda())
    tol = REL_L2 if out == torch.float16 else 1e-5  # bf16 x is exact: only fp32 accumulation remains
    assert R.rel_l2(y.float().cpu().numpy(), R.int8_linear(x.float().numpy(), q, s)) < tol


def test_split_is_exact_and_x2_gemm_matches(sbq):
    # sbq_split_f32_bf16x2: hi = bf16(x), lo = bf16(x - hi) with x - hi exact; the two-part GEMM
    # called directly gives what the drop-in gives
    L = sbq._lib
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    m, k, n = 200, 512, 384
    x = (sbq.workloads.activation(m, k, seed=3, dtype=torch.float32) * 1e3).cuda()
    x[0, :8] = torch.tensor([0.0, -0.0, 1e-30, -3.4e38, 3.4e38, 1.0 + 2 ** -20, 65504.0, 7e-39], device="cuda")
    hi = torch.empty(m, k, dtype=torch.bfloat16, device="cuda")
    lo = torch.empty_like(hi)
    L.call("sbq_split_f32_bf16x2", p(x), k, m, k, p(hi), p(lo), k, st)
    want_hi = x.to(torch.bfloat16)
    assert torch.equal(hi, want_hi)
    assert torch.equal(lo, (x - want_hi.float()).to(torch.bfloat16))
    w = sbq.workloads.float_weight(n, k, seed=4)
    mod = sbq.Int8Linear(w, None)
    x2 = x.clone()
    x2[0, 3:5] = 0.0  # keep the products finite for the output comparison
    L.call("sbq_split_f32_bf16x2", p(x2), k, m, k, p(hi), p(lo), k, st)
    y = torch.empty(m, n, device="cuda")
    L.call("sbq_gemm_w8a16_x2", p(hi), p(lo), k, p(mod.packed), p(mod.scale), None, m, n, k, p(y), L.F32, n, st)
    assert torch.equal(y, mod(x2))


@pytest.mark.parametrize("m", [64, 300])
def test_f32_gated_gateup(sbq, m):
    n, k = 1536, 1024
    wg, wu, wd = (sbq.workloads.float_weight(*sh, seed=m + i) for i, sh in enumerate([(n, k), (n, k), (k, n)]))
    mlp = sbq.FusedGatedMLP(*(sbq.Int8Linear(w, None) for w in (wg, wu, wd)), h_dtype=torch.float32)
    x = sbq.workloads.activation(m, k, seed=m + 4, dtype=torch.float32)
    h = mlp.gateup_into(x.cuda(), torch.empty(m, n, dtype=torch.float32, device="cuda"))
    g, u = (R.int8_linear(x.numpy(), *R.quantize_per_channel(w.numpy())) for w in (wg, wu))
    want = g.astype(np.float64) / (1.0 + np.exp(-g.astype(np.float64))) * u
    assert R.rel_l2(h.cpu().numpy(), want) < 1e-4


def test_f32_workspace_errors_launch_nothing(sbq):
    L = sbq._lib
    lib = L.load()
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    m, n, k = 64, 128, 256
    mod = sbq.Int8Linear(sbq.workloads.float_weight(n, k, seed=1), None)
    x = torch.ones(m, k, device="cuda")
    y = torch.full((m, n), 7.0, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.sbq_linear_w8_ws(p(x), L.F32, k, p(mod.packed), p(mod.scale), None, m, n, k, p(y), L.F32, n, None, 0, st)
    assert rc == L.ERR_INVALID_ARGUMENT
    ws = torch.empty(16, dtype=torch.uint8, device="cuda")
    rc = lib.sbq_linear_w8_ws(p(x), L.F32, k, p(mod.packed), p(mod.scale), None, m, n, k, p(y), L.F32, n, p(ws), 16, st)
    assert rc == L.ERR_WORKSPACE
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())
