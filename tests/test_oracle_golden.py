"""The CPU oracle against the reference's own outputs (tests/golden, made by make_golden.py).

This pins the oracle: weight quantisation and the int8-dyn stages must be
bit-exact with spikingbrain_cpu/quant.py (quant.py:25-29, :63-66); the int8
weight-only forward (quant.py:41-53) must agree with the reference's blocked
fp32 result to fp32 rounding.
"""

import os
import sys

import numpy as np
import pytest

from conftest import cfg3_inputs, golden, golden_cases, golden_cfg3, sha256
from oracle import quant_ref as R


@pytest.mark.parametrize("name", golden_cases())
def test_quantize_per_channel_bit_exact(name):
    g = golden(name)
    q, s = R.quantize_per_channel(g["w"])
    assert np.array_equal(s.view(np.uint32), g["scale"].view(np.uint32))
    assert np.array_equal(q, g["q"])
    qc, sc = R.quantize_per_channel_c(g["w"])
    assert np.array_equal(sc.view(np.uint32), g["scale"].view(np.uint32))
    assert np.array_equal(qc, g["q"])


@pytest.mark.parametrize("name", golden_cases("int8"))
def test_int8_forward_matches_reference(name):
    g = golden(name)
    y = R.int8_linear(g["x"].astype(np.float32), g["q"], g["scale"], g.get("bias"))
    assert y.shape == g["y"].shape
    assert R.rel_l2(y, g["y"]) < 1e-5


@pytest.mark.parametrize("name", golden_cases("int8-dyn"))
def test_dyn_forward_bit_exact(name):
    g = golden(name)
    y, xq, s, zp, acc = R.dyn_linear(g["x"].astype(np.float32), g["q"], g["scale"], g.get("bias"))
    want = g["y"].reshape(y.shape)
    assert np.array_equal(y.view(np.uint32), want.view(np.uint32)), (
        "mismatch fraction %.4f" % float((y != want).mean()))


def test_dyn_rows_subset_consistent():
    g = golden("dyn_m33_n192_k512")
    x = g["x"].astype(np.float32)
    full = R.dyn_linear(x, g["q"], g["scale"])[0]
    rows = np.array([0, 5, 32])
    part = R.dyn_linear(x, g["q"], g["scale"], rows=rows)[0]
    assert np.array_equal(part, full[rows])


def test_qparams_special_cases():
    # all-zero tensor: the scale falls back to 0.1 with zero point 0
    s, zp = R.choose_qparams(0.0, 0.0)
    assert s == np.float32(0.1) and zp == 0
    # positive-only range keeps zero at the bottom of the uint8 range
    s, zp = R.choose_qparams(0.5, 2.0)
    assert zp == 0 and s == np.float32(2.0 / 255.0)
    # negative-only range pins the zero point at 255
    s, zp = R.choose_qparams(-2.0, -0.5)
    assert zp == 255


def test_per_token_mode_restatement():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((7, 96)).astype(np.float32)
    x[3] = 0.0
    w = (rng.standard_normal((24, 96)) * 0.02).astype(np.float32)
    q, scale = R.quantize_per_channel(w)
    y, xq, s_tok, acc = R.tok_linear(x, q, scale)
    assert s_tok[3] == np.float32(1e-8) / np.float32(127.0) and not xq[3].any()
    assert np.abs(xq).max() <= 127
    ref = acc.astype(np.int64)
    assert np.array_equal(ref, xq.astype(np.int64) @ q.astype(np.int64).T)
    # the per-token result approximates the float product
    assert R.rel_l2(y, R.int8_linear(x, q, scale)) < 2e-2


def test_config3_oracle_matches_reference_digests():
    # benchmark configuration 3 (int8-dyn, m=512, k=n=4096): the oracle reproduces every output of
    # the reference's DynamicInt8Linear bit for bit (digests made by make_golden.py from the reference)
    ref = golden_cfg3()
    w, x = cfg3_inputs()
    assert sha256(w.numpy()) == ref["w_sha256"] and sha256(x.numpy()) == ref["x_sha256"], \
        "the seeded inputs differ on this machine (torch generator), so the digests cannot be compared"
    q, scale = R.quantize_per_channel(w.numpy())
    assert sha256(q) == ref["q_sha256"] and sha256(scale) == ref["scale_sha256"]
    y, xq, s, zp, acc = R.dyn_linear(x.float().numpy(), q, scale)
    assert int(np.float32(s).view(np.uint32)) == ref["s_x_bits"] and zp == ref["zp"]
    assert sha256(xq) == ref["xq_sha256"]
    assert np.array_equal(y[ref["rows"]].view(np.uint32), ref["y_rows"].view(np.uint32))
    assert sha256(y) == ref["y_sha256"]


@pytest.mark.skipif(not os.environ.get("SBQ_REFERENCE_ROOT"),
                    reason="set SBQ_REFERENCE_ROOT to the reference's root directory to re-run it here")
@pytest.mark.parametrize("m,n,k,seed", [(512, 4096, 4096, 5), (77, 300, 2560, 6), (1, 64, 128, 7)])
def test_oracle_matches_live_reference(m, n, k, seed):
    # the reference itself (its quant.py, fbgemm engine x86) on fresh seeded inputs, against the
    # oracle: weight quantisation and the int8-dyn output bit for bit, the int8 output to fp32 rounding
    import torch

    sys.path.insert(0, os.environ["SBQ_REFERENCE_ROOT"])
    from spikingbrain_cpu import quant

    torch.backends.quantized.engine = "x86"
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(n, k, generator=g) * 0.02
    x = torch.randn(m, k, generator=g) * 1.5 + 0.1
    q, s = R.quantize_per_channel(w.numpy())
    rq, rs = quant.quantize_per_channel(w)
    assert np.array_equal(q, rq.numpy()) and np.array_equal(s.view(np.uint32), rs.numpy().view(np.uint32))
    y = R.dyn_linear(x.numpy(), q, s)[0]
    ry = quant.DynamicInt8Linear(w, None)(x).numpy()
    assert np.array_equal(y.view(np.uint32), ry.view(np.uint32))
    assert R.rel_l2(R.int8_linear(x.numpy(), q, s), quant.Int8Linear(w, None)(x).numpy()) < 1e-5
