"""GPU parity of the int8 weight-only path (format "int8") against the CPU oracle and the
reference's golden outputs.

Tolerances (stated by the north star): weight quantisation bit-exact; fp32/fp16 outputs within a
relative L2 error of 1e-3 of quant.py (Int8Linear.forward, quant.py:41-53).
"""

import numpy as np
import pytest
import torch

from conftest import golden, golden_cases
from oracle import quant_ref as R

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3


def _np(t):
    return t.detach().float().cpu().numpy() if t.dtype in (torch.float16, torch.bfloat16) else t.detach().cpu().numpy()


@pytest.mark.parametrize("name", golden_cases())
def test_device_quantisation_bit_exact(sbq, name):
    g = golden(name)
    w = torch.from_numpy(g["w"])
    if g["meta"]["w_dtype"] == "bfloat16":
        w = w.to(torch.bfloat16)
    q, s = sbq.quantize_per_channel(w)
    assert np.array_equal(q.cpu().numpy(), g["q"])
    assert np.array_equal(s.cpu().numpy().view(np.uint32), g["scale"].view(np.uint32))


@pytest.mark.parametrize("name", golden_cases("int8"))
def test_int8_linear_matches_reference_golden(sbq, name):
    g = golden(name)
    w = torch.from_numpy(g["w"])
    if g["meta"]["w_dtype"] == "bfloat16":
        w = w.to(torch.bfloat16)
    bias = torch.from_numpy(g["bias"]) if "bias" in g else None
    x = torch.from_numpy(g["x"])
    if g["meta"]["x_dtype"] == "bfloat16":
        x = x.to(torch.bfloat16)
    mod = sbq.Int8Linear(w, bias)
    y = mod(x.cuda())
    assert y.dtype == torch.float32 and tuple(y.shape) == g["y"].shape
    assert R.rel_l2(_np(y), g["y"]) < REL_L2


@pytest.mark.parametrize("m", [1, 2, 3, 7, 8, 9, 15, 16, 17, 33])
@pytest.mark.parametrize("xdtype", [torch.float16, torch.bfloat16, torch.float32])
def test_gemv_odd_shapes_vs_oracle(sbq, m, xdtype):
    n, k = 130, 320
    w = sbq.workloads.float_weight(n, k, seed=100 + m)
    x = sbq.workloads.activation(m, k, seed=200 + m, dtype=xdtype)
    q, s = R.quantize_per_channel(w.numpy())
    mod = sbq.Int8Linear(w, None)
    y = mod(x.cuda())
    want = R.int8_linear(x.float().numpy(), q, s)
    tol = 2e-5 if xdtype == torch.float32 else REL_L2
    assert R.rel_l2(_np(y), want) < tol


@pytest.mark.parametrize("n,k", [(4, 2560), (64, 2560), (128, 128), (1024, 2560), (4096, 4096), (4096, 12288),
                                 (12288, 4096), (200, 64)])
def test_gemv_model_shapes(sbq, n, k):
    w = sbq.workloads.float_weight(n, k, seed=n + k)
    x = sbq.workloads.activation(1, k, seed=7)
    q, s = R.quantize_per_channel(w.numpy())
    y = sbq.Int8Linear(w, None)(x.cuda())
    assert R.rel_l2(_np(y), R.int8_linear(x.float().numpy(), q, s)) < REL_L2


def test_config0_decode_gemv(sbq):
    cfg = sbq.workloads.CONFIGS[0]
    w = sbq.workloads.float_weight(cfg["n"], cfg["k"], seed=0)
    x = sbq.workloads.activation(cfg["m"], cfg["k"], seed=1)
    q, s = R.quantize_per_channel(w.numpy())
    mod = sbq.Int8Linear(w, None)
    assert torch.equal(mod.qweight.cpu(), torch.from_numpy(q))
    y = mod(x.cuda())
    assert R.rel_l2(_np(y), R.int8_linear(x.float().numpy(), q, s)) < REL_L2


def test_fp16_output_and_bias(sbq):
    n, k, m = 96, 256, 5
    w = sbq.workloads.float_weight(n, k, seed=3)
    b = torch.randn(n)
    x = sbq.workloads.activation(m, k, seed=4)
    q, s = R.quantize_per_channel(w.numpy())
    mod = sbq.Int8Linear(w, b)
    mod.out_dtype = torch.float16
    y = mod(x.cuda())
    assert y.dtype == torch.float16
    assert R.rel_l2(_np(y), R.int8_linear(x.float().numpy(), q, s, b.numpy())) < REL_L2


def test_host_input_returns_host_output(sbq):
    w = sbq.workloads.float_weight(64, 128, seed=5)
    x = sbq.workloads.activation(3, 128, seed=6, dtype=torch.float32)
    y = sbq.Int8Linear(w, None)(x)
    assert y.device.type == "cpu"
    q, s = R.quantize_per_channel(w.numpy())
    assert R.rel_l2(y.numpy(), R.int8_linear(x.numpy(), q, s)) < 2e-5


def test_empty_and_batched_inputs(sbq):
    w = sbq.workloads.float_weight(32, 64, seed=8)
    mod = sbq.Int8Linear(w, None)
    y = mod(torch.zeros(0, 64, device="cuda", dtype=torch.float16))
    assert tuple(y.shape) == (0, 32)
    x = sbq.workloads.activation(6, 64, seed=9).reshape(2, 3, 64)
    y = mod(x.cuda())
    assert tuple(y.shape) == (2, 3, 32)
    q, s = R.quantize_per_channel(w.numpy())
    assert R.rel_l2(_np(y).reshape(6, 32), R.int8_linear(x.float().numpy().reshape(6, 64), q, s)) < REL_L2


def test_k_not_multiple_of_16(sbq):
    w = sbq.workloads.float_weight(40, 77, seed=10)
    x = sbq.workloads.activation(4, 77, seed=11, dtype=torch.float32)
    q, s = R.quantize_per_channel(w.numpy())
    y = sbq.Int8Linear(w, None)(x.cuda())
    assert R.rel_l2(_np(y), R.int8_linear(x.numpy(), q, s)) < 2e-5


def test_state_dict_round_trip(sbq):
    w = sbq.workloads.float_weight(48, 128, seed=12)
    a = sbq.Int8Linear(w, None)
    sd = a.state_dict()
    assert set(sd) == {"qweight", "scale"} and sd["qweight"].dtype == torch.int8
    b = sbq.Int8Linear(torch.zeros(48, 128), None)
    b.load_state_dict(sd)
    x = sbq.workloads.activation(2, 128, seed=13).cuda()
    assert torch.equal(a(x), b(x))


def test_pack_unpack_round_trip(sbq):
    q = torch.randint(-127, 128, (33, 200), dtype=torch.int8)
    packed, rs = sbq.pack_int8(q, rowsum=True)
    assert torch.equal(sbq.unpack_int8(packed, 33, 200).cpu(), q)
    assert torch.equal(rs.cpu(), q.int().sum(1).int())


@pytest.mark.parametrize("m", [1, 4, 16])
def test_fused_gateup_mlp_vs_oracle(sbq, m):
    n, k = 1024, 512
    wg = sbq.workloads.float_weight(n, k, seed=20)
    wu = sbq.workloads.float_weight(n, k, seed=21)
    wd = sbq.workloads.float_weight(k, n, seed=22)
    x = sbq.workloads.activation(m, k, seed=23)
    gate, up, down = (sbq.Int8Linear(w, None) for w in (wg, wu, wd))
    mlp = sbq.FusedGatedMLP(gate, up, down)
    y = mlp(x.cuda())
    o = [R.quantize_per_channel(w.numpy()) for w in (wg, wu, wd)]
    want = R.gated_mlp(x.float().numpy(), o[0], o[1], o[2])
    assert R.rel_l2(_np(y), want) < REL_L2
    # the unfused reference composition gives the same answer
    ref = down(torch.nn.functional.silu(gate(x.cuda())) * up(x.cuda()))
    assert R.rel_l2(_np(y), _np(ref)) < REL_L2


@pytest.mark.parametrize("m", [1, 5, 16])
def test_grouped_launch_matches_single_calls(sbq, m):
    from importlib import import_module
    quant = import_module("spikingbrain-cpu_b200.quant")
    k = 512
    a = sbq.Int8Linear(sbq.workloads.float_weight(384, k, seed=80), torch.randn(384))
    b = sbq.Int8Linear(sbq.workloads.float_weight(200, k, seed=81), None)
    mlp = sbq.FusedGatedMLP(*(sbq.Int8Linear(sbq.workloads.float_weight(*sh, seed=82 + i), None)
                              for i, sh in enumerate([(256, k), (256, k), (k, 256)])))
    x = sbq.workloads.activation(m, k, seed=85).cuda()
    ya, yb = torch.empty(m, 384, device="cuda"), torch.empty(m, 200, device="cuda", dtype=torch.float16)
    h = torch.empty(m, 256, device="cuda", dtype=torch.float16)
    quant.gemv_group([mlp.gateup_job(x, h), a.gemv_job(x, ya), b.gemv_job(x, yb)], x.dtype, m, x.device)
    b.out_dtype = torch.float16
    assert torch.equal(ya, a(x)) and torch.equal(yb, b(x))
    assert torch.equal(h, mlp.gateup_into(x, torch.empty_like(h)))


@pytest.mark.parametrize("n,k,m", [(64, 12288, 1), (256, 12288, 3), (1024, 8192, 12), (96, 4096, 5)])
@pytest.mark.parametrize("out", [torch.float32, torch.float16])
def test_split_k_gemv_vs_oracle(sbq, n, k, m, out):
    # few row tiles with long K: the launch cuts each tile into K parts whose partial sums are
    # added in part order by the CTA that completes the tile (deterministic)
    w = sbq.workloads.float_weight(n, k, seed=n + 3 * k)
    b = torch.randn(n)
    x = sbq.workloads.activation(m, k, seed=m + 40)
    q, s = R.quantize_per_channel(w.numpy())
    mod = sbq.Int8Linear(w, b)
    mod.out_dtype = out
    y1 = mod(x.cuda())
    y2 = mod(x.cuda())
    assert torch.equal(y1, y2)
    assert R.rel_l2(_np(y1), R.int8_linear(x.float().numpy(), q, s, b.numpy())) < REL_L2


@pytest.mark.parametrize("xdtype", [torch.bfloat16, torch.float32])
def test_split_k_other_activation_types(sbq, xdtype):
    n, k, m = 128, 12288, 2
    w = sbq.workloads.float_weight(n, k, seed=51)
    x = sbq.workloads.activation(m, k, seed=52, dtype=xdtype)
    q, s = R.quantize_per_channel(w.numpy())
    y = sbq.Int8Linear(w, None)(x.cuda())
    tol = 2e-5 if xdtype == torch.float32 else REL_L2
    assert R.rel_l2(_np(y), R.int8_linear(x.float().numpy(), q, s)) < tol


@pytest.mark.parametrize("m", [1, 6])
def test_split_k_fused_gateup(sbq, m):
    n, k = 64, 8192
    wg = sbq.workloads.float_weight(n, k, seed=60)
    wu = sbq.workloads.float_weight(n, k, seed=61)
    wd = sbq.workloads.float_weight(k, n, seed=62)
    x = sbq.workloads.activation(m, k, seed=63)
    mlp = sbq.FusedGatedMLP(*(sbq.Int8Linear(w, None) for w in (wg, wu, wd)))
    h1 = mlp.gateup_into(x.cuda(), torch.empty(m, n, device="cuda"))
    h2 = mlp.gateup_into(x.cuda(), torch.empty(m, n, device="cuda"))
    assert torch.equal(h1, h2)
    g, u = (R.int8_linear(x.float().numpy(), *R.quantize_per_channel(w.numpy())) for w in (wg, wu))
    want = g / (1.0 + np.exp(-g)) * u
    assert R.rel_l2(_np(h1), want) < REL_L2


# The checkpoint's projection shapes (hidden 2560, 32 heads of 128, 8 key/value heads, MLP 9728,
# vocabulary 151936; spikingbrain_cpu/model.py:232-301 and the tied head, loader.py:94), as [N, K].
REAL_SHAPES = [(9728, 2560), (2560, 9728), (4096, 2560), (1024, 2560), (2560, 4096), (128, 2560), (4096, 128),
               (64, 2560), (4, 2560)]


@pytest.mark.parametrize("n,k", REAL_SHAPES)
@pytest.mark.parametrize("m", [1, 7, 100])
def test_real_model_shapes_vs_oracle(sbq, n, k, m):
    # fp32 activations, as the reference's model passes them (quant.py:47)
    w = sbq.workloads.float_weight(n, k, seed=n * 7 + k)
    x = sbq.workloads.activation(m, k, seed=m + n, dtype=torch.float32)
    q, s = R.quantize_per_channel(w.numpy())
    y = sbq.Int8Linear(w, None)(x.cuda())
    assert R.rel_l2(_np(y), R.int8_linear(x.numpy(), q, s)) < 2e-5


def test_tied_head_shape(sbq):
    # the [151936 x 2560] int8 head at decode, checked on the first and last 1024 rows
    n, k = 151936, 2560
    w = sbq.workloads.float_weight(n, k, seed=9)
    x = sbq.workloads.activation(1, k, seed=10)
    y = _np(sbq.Int8Linear(w, None)(x.cuda()))
    for rows in (slice(0, 1024), slice(n - 1024, n)):
        q, s = R.quantize_per_channel(w[rows].numpy())
        assert R.rel_l2(y[:, rows], R.int8_linear(x.float().numpy(), q, s)) < REL_L2


def test_shared_input_projection_group(sbq):
    # sse_q/k/v and swa_q/k/v of one hybrid block read the same x (model.py:317-321, :363-365): one
    # grouped launch gives what six separate calls give
    from importlib import import_module
    quant = import_module("spikingbrain-cpu_b200.quant")
    hid = 2560
    mods = [sbq.Int8Linear(sbq.workloads.float_weight(n, hid, seed=90 + i), None)
            for i, n in enumerate((4096, 4096, 4096, 4096, 1024, 1024))]
    x = sbq.workloads.activation(1, hid, seed=99).cuda()
    outs = [torch.empty(1, mod.out_features, device="cuda") for mod in mods]
    quant.gemv_group([mod.gemv_job(x, o) for mod, o in zip(mods, outs)], x.dtype, 1, x.device)
    for mod, o in zip(mods, outs):
        assert torch.equal(o, mod(x))


def test_lora_projection_pair(sbq):
    # lora_q_proj = Linear(2560 -> 128) then Linear(128 -> 4096) (model.py:287)
    a = sbq.workloads.float_weight(128, 2560, seed=77)
    b = sbq.workloads.float_weight(4096, 128, seed=78)
    x = sbq.workloads.activation(3, 2560, seed=79, dtype=torch.float32)
    la, lb = sbq.Int8Linear(a, None), sbq.Int8Linear(b, None)
    y = lb(la(x.cuda()))
    qa, sa = R.quantize_per_channel(a.numpy())
    qb, sb = R.quantize_per_channel(b.numpy())
    want = R.int8_linear(R.int8_linear(x.numpy(), qa, sa).astype(np.float32), qb, sb)
    assert R.rel_l2(_np(y), want) < 1e-4
