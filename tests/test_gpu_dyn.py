"""GPU parity of the int8-dyn path (DynamicInt8Linear, spikingbrain_cpu/quant.py:56-66).

The north star's bar: bit-exact int32 accumulators and quantised activations, and (since the
epilogue is restated exactly) bit-exact fp32 outputs, against the reference's golden outputs and
the oracle's integer stages.
"""

import numpy as np
import pytest
import torch

from conftest import cfg3_inputs, golden, golden_cases, golden_cfg3, sha256
from oracle import quant_ref as R

pytestmark = pytest.mark.gpu


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def _x_tensor(g):
    x = torch.from_numpy(g["x"])
    if g["meta"]["x_dtype"] == "bfloat16":
        x = x.to(torch.bfloat16)
    return x


@pytest.mark.parametrize("name", golden_cases("int8-dyn"))
def test_dyn_matches_reference_golden_bit_exact(sbq, name):
    g = golden(name)
    bias = torch.from_numpy(g["bias"]) if "bias" in g else None
    mod = sbq.DynamicInt8Linear(torch.from_numpy(g["w"]), bias)
    y = mod(_x_tensor(g).cuda())
    assert tuple(y.shape) == g["y"].shape
    got = y.cpu().numpy()
    assert np.array_equal(_bits(got), _bits(g["y"])), "mismatch fraction %.4f" % float((got != g["y"]).mean())


@pytest.mark.parametrize("name", golden_cases("int8-dyn"))
def test_dyn_integer_stages_bit_exact(sbq, name):
    g = golden(name)
    bias = torch.from_numpy(g["bias"]) if "bias" in g else None
    mod = sbq.DynamicInt8Linear(torch.from_numpy(g["w"]), bias)
    x = _x_tensor(g)
    y, xq, s, zp, acc = mod.forward_stages(x.cuda())
    ry, rxq, rs, rzp, racc = R.dyn_linear(x.float().numpy().reshape(-1, x.shape[-1]), g["q"], g["scale"], g.get("bias"))
    assert float(s.item()) == float(rs) and int(zp.item()) == rzp
    assert np.array_equal(xq.cpu().numpy(), rxq)
    assert np.array_equal(acc.cpu().numpy(), racc)
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(ry))


def test_config3_full_size(sbq):
    cfg = sbq.workloads.CONFIGS[3]
    m, k, n = cfg["m"], cfg["k"], cfg["n"]
    w = sbq.workloads.float_weight(n, k, seed=30)
    x = sbq.workloads.activation(m, k, seed=31)  # fp16 N(0, 1), the configuration's input
    q, sc = R.quantize_per_channel(w.numpy())
    mod = sbq.DynamicInt8Linear(w, None)
    y, xq, s, zp, acc = mod.forward_stages(x.cuda())
    rows = np.array([0, 1, 77, 128, 255, 256, 383, 510, 511])
    ry, rxq, rs, rzp, racc = R.dyn_linear(x.float().numpy(), q, sc, rows=rows)
    assert float(s.item()) == float(rs) and int(zp.item()) == rzp
    # every quantised activation, and the sampled rows' accumulators and outputs
    full_xq = R.dyn_quantize(x.float().numpy(), rs, rzp)
    assert np.array_equal(xq.cpu().numpy(), full_xq)
    assert np.array_equal(acc.cpu().numpy()[rows], racc)
    assert np.array_equal(_bits(y.cpu().numpy()[rows]), _bits(ry))
    # forward() (fused workspace path) gives the same output as the staged path
    assert torch.equal(mod(x.cuda()), y)
    assert sbq._lib.load().sbq_check_device_error() == 0


@pytest.mark.parametrize("path", ["forward", "stages"])
def test_config3_matches_reference_digests(sbq, path):
    # configuration 3 at full size against the reference's own outputs (digests of the whole
    # quantised activation and of the whole fp32 output, made by running the reference's
    # DynamicInt8Linear): bit-exact on every element, the oracle not involved
    ref = golden_cfg3()
    w, x = cfg3_inputs()
    assert sha256(w.numpy()) == ref["w_sha256"] and sha256(x.numpy()) == ref["x_sha256"], \
        "the seeded inputs differ on this machine (torch generator), so the digests cannot be compared"
    mod = sbq.DynamicInt8Linear(w, None)
    assert sha256(mod.qweight.cpu().numpy()) == ref["q_sha256"]
    assert sha256(mod.scale.cpu().numpy()) == ref["scale_sha256"]
    if path == "forward":
        y = mod(x.cuda()).cpu().numpy()
    else:
        yt, xq, s, zp, _ = mod.forward_stages(x.cuda())
        y = yt.cpu().numpy()
        assert sha256(xq.cpu().numpy()) == ref["xq_sha256"]
        assert int(s.cpu().numpy().view(np.uint32)[0]) == ref["s_x_bits"] and int(zp.item()) == ref["zp"]
    assert np.array_equal(y[ref["rows"]].view(np.uint32), ref["y_rows"].view(np.uint32))
    assert sha256(y) == ref["y_sha256"]


@pytest.mark.parametrize("m,n,k", [(1, 4, 64), (3, 40, 192), (127, 130, 320), (129, 300, 256), (200, 64, 2560),
                                   (257, 4096, 128), (64, 1024, 2560)])
@pytest.mark.parametrize("xdtype", [torch.float32, torch.float16, torch.bfloat16])
def test_dyn_shapes_bit_exact(sbq, m, n, k, xdtype):
    w = sbq.workloads.float_weight(n, k, seed=m + n)
    x = sbq.workloads.activation(m, k, seed=k, dtype=xdtype) * 2.5
    q, sc = R.quantize_per_channel(w.numpy())
    mod = sbq.DynamicInt8Linear(w, None)
    y = mod(x.cuda()).cpu().numpy()
    ry = R.dyn_linear(x.float().numpy(), q, sc)[0]
    assert np.array_equal(_bits(y), _bits(ry)), "mismatch fraction %.4f" % float((y != ry).mean())


@pytest.mark.parametrize("m,n,k,xdtype", [(1, 64, 128, torch.float32), (5, 130, 320, torch.float32),
                                          (128, 256, 512, torch.float32), (300, 200, 1024, torch.float32),
                                          # rows longer than the per-thread register cache (512 vectors):
                                          # the two-pass path that reads each row twice
                                          (3, 96, 2560, torch.float32), (4, 64, 4160, torch.float16)])
def test_per_token_mode_bit_exact(sbq, m, n, k, xdtype):
    w = sbq.workloads.float_weight(n, k, seed=n)
    x = sbq.workloads.activation(m, k, seed=m, dtype=torch.float32)
    x[0] = 0.0  # an all-zero token takes the 1e-8 floor
    x = x.to(xdtype)
    q, sc = R.quantize_per_channel(w.numpy())
    mod = sbq.DynamicInt8Linear(w, None, mode="per_token")
    y, xq, s, _, acc = mod.forward_stages(x.cuda())
    ry, rxq, rs, racc = R.tok_linear(x.float().numpy(), q, sc)
    assert np.array_equal(_bits(s.cpu().numpy()), _bits(rs))
    assert np.array_equal(xq.cpu().numpy(), rxq)
    assert np.array_equal(acc.cpu().numpy(), racc)
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(ry))
    assert torch.equal(mod(x.cuda()), y)


def test_dyn_host_input_and_batch_dims(sbq):
    w = sbq.workloads.float_weight(48, 128, seed=40)
    x = sbq.workloads.activation(6, 128, seed=41, dtype=torch.float32).reshape(2, 3, 128)
    mod = sbq.DynamicInt8Linear(w, None)
    y = mod(x)
    assert y.device.type == "cpu" and tuple(y.shape) == (2, 3, 48)
    q, sc = R.quantize_per_channel(w.numpy())
    assert np.array_equal(_bits(y.numpy().reshape(6, 48)), _bits(R.dyn_linear(x.numpy().reshape(6, 128), q, sc)[0]))


@pytest.mark.parametrize("ldy_pad", [4, 1, 36])
@pytest.mark.parametrize("mode", ["per_tensor", "per_token"])
def test_dyn_strided_output_rows(sbq, ldy_pad, mode):
    """y with a row stride above n, 16-byte aligned rows (staged tile stores) or not (direct stores);
    the padding columns between rows stay untouched."""
    import ctypes

    m, n, k = 200, 300, 512
    w = sbq.workloads.float_weight(n, k, seed=60)
    x = sbq.workloads.activation(m, k, seed=61, dtype=torch.float16).cuda()
    mod = sbq.DynamicInt8Linear(w, None, mode=mode)
    want = mod(x)
    L = sbq._lib
    ldy = n + ldy_pad
    y = torch.full((m, ldy), -7.25, device="cuda")
    code = L.ACT_PER_TENSOR if mode == "per_tensor" else L.ACT_PER_TOKEN
    wsb = int(L.load().sbq_dyn_workspace_bytes(m, k, code))
    ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
    p = lambda t: None if t is None else ctypes.c_void_p(t.data_ptr())  # noqa: E731
    L.call("sbq_linear_dyn", p(x), L.F16, k, code, p(mod.packed), p(mod.rowsum), p(mod.scale), None, m, n, k, p(y),
           ldy, p(ws), wsb, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert torch.equal(y[:, :n], want)
    assert bool((y[:, n:] == -7.25).all())
    assert sbq._lib.load().sbq_check_device_error() == 0


# x of 8 MiB and more takes the one-launch quantiser (grid barrier): with the whole of x held in
# registers (cached) or, above what the grid's registers hold, read twice; dense and strided rows.
@pytest.mark.parametrize("m,k,xdtype,ld_pad", [(1024, 2048, torch.float32, 0), (1100, 4096, torch.float16, 0),
                                               (1200, 4096, torch.float32, 0), (2400, 4096, torch.bfloat16, 0),
                                               (1100, 2048, torch.float32, 64)])
def test_one_launch_quantiser_bit_exact(sbq, m, k, xdtype, ld_pad):
    import ctypes

    n = 64
    w = sbq.workloads.float_weight(n, k, seed=m)
    x = (sbq.workloads.activation(m, k, seed=k + m, dtype=torch.float32) * 3.0).to(xdtype)
    x[7, 5] = 40.0  # an outlier that sets the range
    q, sc = R.quantize_per_channel(w.numpy())
    ry, rxq, rs, rzp, racc = R.dyn_linear(x.float().numpy(), q, sc)
    mod = sbq.DynamicInt8Linear(w, None)
    if ld_pad == 0:
        y, xq, s, zp, acc = mod.forward_stages(x.cuda())
        assert np.array_equal(acc.cpu().numpy(), racc)
    else:
        xs = torch.zeros(m, k + ld_pad, dtype=xdtype)
        xs[:, :k] = x
        xs = xs.cuda()
        L = sbq._lib
        dt = {torch.float32: L.F32, torch.float16: L.F16, torch.bfloat16: L.BF16}[xdtype]
        wsb = int(L.load().sbq_dyn_workspace_bytes(m, k, L.ACT_PER_TENSOR))
        ws = torch.empty(wsb, dtype=torch.uint8, device="cuda")
        xq = torch.empty(m, k, dtype=torch.uint8, device="cuda")
        s = torch.empty(1, device="cuda")
        zp = torch.empty(1, dtype=torch.int32, device="cuda")
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        L.call("sbq_quant_act_per_tensor", p(xs), dt, k + ld_pad, m, k, p(xq), p(s), p(zp), p(ws), wsb,
               ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        y = torch.empty(m, n, device="cuda")
        L.call("sbq_linear_dyn", p(xs), dt, k + ld_pad, L.ACT_PER_TENSOR, p(mod.packed), p(mod.rowsum), p(mod.scale),
               None, m, n, k, p(y), n, p(ws), wsb, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert float(s.item()) == float(rs) and int(zp.item()) == rzp
    assert np.array_equal(xq.cpu().numpy(), rxq)
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(ry))
    assert sbq._lib.load().sbq_check_device_error() == 0


def test_one_launch_quantiser_repeated_and_alternating(sbq):
    """The grid barrier's counters are reused launch after launch (and by launches of other sizes in
    between, which take the other path or another grid size): results stay bit-identical."""
    w = sbq.workloads.float_weight(64, 4096, seed=3)
    mod = sbq.DynamicInt8Linear(w, None)
    big = sbq.workloads.activation(1024, 4096, seed=4, dtype=torch.float32).cuda()  # 16 MiB: re-read path
    mid = sbq.workloads.activation(600, 4096, seed=5, dtype=torch.float32).cuda()   # 9.4 MiB: cached
    small = sbq.workloads.activation(40, 4096, seed=6, dtype=torch.float32).cuda()  # two-kernel path
    want = [mod(t) for t in (big, mid, small)]
    for _ in range(5):
        for t, wv in zip((big, mid, small), want):
            assert torch.equal(mod(t), wv)
    assert sbq._lib.load().sbq_check_device_error() == 0


# decode sizes (up to 32 rows): K split over a cluster of CTAs (int32 partial sums added in the owning
# CTA); bit-exact like every other int8-dyn path, per tensor and per token, with and without bias;
# 33 rows takes the unsplit kernel
@pytest.mark.parametrize("m,n,k", [(1, 4096, 4096), (16, 4096, 4096), (5, 1000, 2560), (32, 512, 1024),
                                   (33, 512, 1024)])
@pytest.mark.parametrize("mode", ["per_tensor", "per_token"])
def test_decode_split_k_bit_exact(sbq, m, n, k, mode):
    w = sbq.workloads.float_weight(n, k, seed=n + m)
    bias = torch.randn(n) if m % 2 else None
    x = sbq.workloads.activation(m, k, seed=k + m, dtype=torch.float32) * 2.0
    q, sc = R.quantize_per_channel(w.numpy())
    mod = sbq.DynamicInt8Linear(w, bias, mode=mode)
    y, xq, s, _, acc = mod.forward_stages(x.cuda())
    b = None if bias is None else bias.numpy()
    if mode == "per_tensor":
        ry, rxq, rs, rzp, racc = R.dyn_linear(x.numpy(), q, sc, b)
    else:
        ry, rxq, rs, racc = R.tok_linear(x.numpy(), q, sc, b)
    assert np.array_equal(xq.cpu().numpy(), rxq)
    assert np.array_equal(acc.cpu().numpy(), racc)
    assert np.array_equal(_bits(y.cpu().numpy()), _bits(ry))
    assert torch.equal(mod(x.cuda()), y)
    assert sbq._lib.load().sbq_check_device_error() == 0


# decode-sized calls through the module (one-CTA quantiser, split-K GEMM): k not a multiple of 128
# leaves a ragged last k-block; x rows with a stride above k; an all-zero token; the largest k.
@pytest.mark.parametrize("m,n,k", [(1, 256, 144), (2, 136, 4112), (7, 1000, 2560), (8, 4096, 12288),
                                   (9, 300, 512), (1, 64, 12304)])
@pytest.mark.parametrize("xdtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("mode", ["per_tensor", "per_token"])
def test_decode_sizes_ragged_k_strided_rows_bit_exact(sbq, m, n, k, xdtype, mode):
    w = sbq.workloads.float_weight(n, k, seed=n + k)
    bias = torch.randn(n) if m % 2 else None
    wide = sbq.workloads.activation(m, k + 64, seed=m + k, dtype=torch.float32) * 3.0
    if m > 1:
        wide[-1] = 0.0
    x = wide.to(xdtype).cuda()[:, 32:32 + k]  # 16-byte aligned rows, row stride k + 64
    assert x.stride(0) == k + 64
    q, sc = R.quantize_per_channel(w.numpy())
    mod = sbq.DynamicInt8Linear(w, bias, mode=mode)
    y = mod(x).cpu().numpy()
    xf = x.float().cpu().numpy()
    b = None if bias is None else bias.numpy()
    ry = R.dyn_linear(xf, q, sc, b)[0] if mode == "per_tensor" else R.tok_linear(xf, q, sc, b)[0]
    assert np.array_equal(_bits(y), _bits(ry)), "mismatch fraction %.4f" % float((y != ry).mean())
    assert sbq._lib.load().sbq_check_device_error() == 0
