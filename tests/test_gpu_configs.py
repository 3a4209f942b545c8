"""GPU parity at the benchmark configurations' own shapes (configurations 0, 1, 2 and 4).

The oracle is the float64 restatement of Int8Linear.forward (spikingbrain_cpu/quant.py:41-53) and
GatedMLP.forward (model.py:239-240).  Tolerance: relative L2 1e-3, the north star's bar for the
int8 weight-only format.  Where the oracle cannot afford every output row, the rows it checks cover
every M tile of the kernel, and two size-independent checks cover every element: the column sums
of the output against (sum of the activation rows) x W^T x scale, and the row sums against
x . (sum over channels of scale[n] q[n, :]) - both follow from linearity, so a wrong tile anywhere
shows up in them.
"""

import numpy as np
import pytest
import torch

from oracle import quant_ref as R

pytestmark = pytest.mark.gpu

REL_L2 = 1e-3


def _np(t):
    return t.detach().float().cpu().numpy()


def _linearity_checks(x: np.ndarray, y: np.ndarray, q: np.ndarray, s: np.ndarray):
    """Column and row sums of y = (x q^T) * s against the exact sums (float64)."""
    x64, y64 = x.astype(np.float64), y.astype(np.float64)
    col_want = (x64.sum(0) @ q.T.astype(np.float64)) * s.astype(np.float64)
    assert R.rel_l2(y64.sum(0), col_want) < REL_L2
    row_want = x64 @ (q.astype(np.float64) * s.astype(np.float64)[:, None]).sum(0)
    # a row sum adds n outputs of random sign: compare against the scale of the summed terms
    err = np.abs(y64.sum(1) - row_want)
    assert float(err.max()) < REL_L2 * float(np.sqrt((y64 ** 2).sum(1)).max() + 1e-30) * 4


def test_config0_full_output(sbq):
    cfg = sbq.workloads.CONFIGS[0]
    w = sbq.workloads.float_weight(cfg["n"], cfg["k"], seed=0)
    x = sbq.workloads.activation(cfg["m"], cfg["k"], seed=1)
    q, s = R.quantize_per_channel(w.numpy())
    y = sbq.Int8Linear(w, None)(x.cuda())
    assert y.dtype == torch.float32 and tuple(y.shape) == (1, cfg["n"])
    assert R.rel_l2(_np(y), R.int8_linear(x.float().numpy(), q, s)) < REL_L2


@pytest.fixture(scope="module")
def cfg1_weights(sbq):
    cfg = sbq.workloads.CONFIGS[1]
    k, n = cfg["k"], cfg["n"]
    ws = [sbq.workloads.float_weight(*sh, seed=110 + i) for i, sh in enumerate([(n, k), (n, k), (k, n)])]
    mods = [sbq.Int8Linear(w, None) for w in ws]
    oracle = [R.quantize_per_channel(w.numpy()) for w in ws]
    return mods, oracle


@pytest.mark.parametrize("m", [1, 4, 16])
def test_config1_fused_mlp_full_shape(sbq, cfg1_weights, m):
    # gate/up [12288 x 4096], down [4096 x 12288]: the fused gate/up GEMV writes h once in fp16
    # (SiLU(gate) * up in its epilogue), then the down GEMV; every output element is compared
    mods, o = cfg1_weights
    mlp = sbq.FusedGatedMLP(*mods)
    x = sbq.workloads.activation(m, mods[0].in_features, seed=120 + m)
    y = mlp(x.cuda())
    assert tuple(y.shape) == (m, mods[2].out_features)
    want = R.gated_mlp(x.float().numpy(), o[0], o[1], o[2], h_dtype=np.float16)
    assert R.rel_l2(_np(y), want) < REL_L2
    # h itself, every element of [m, 12288]
    h = mlp.gateup_into(x.cuda(), torch.empty(m, mods[0].out_features, dtype=torch.float16, device="cuda"))
    g = R.int8_linear(x.float().numpy(), *o[0])
    u = R.int8_linear(x.float().numpy(), *o[1])
    assert R.rel_l2(_np(h), R.silu(g) * u) < REL_L2


def test_config2_every_m_tile(sbq):
    # m=2048 tokens, k=4096, n=12288, fp16 out: the kernel computes 256-token x 128-channel tiles;
    # the oracle checks the first, middle and last rows of every 256-token tile in full (all 96
    # channel tiles), and the linearity checks cover every element
    cfg = sbq.workloads.CONFIGS[2]
    m, k, n = cfg["m"], cfg["k"], cfg["n"]
    w = sbq.workloads.float_weight(n, k, seed=50)
    x = sbq.workloads.activation(m, k, seed=51)
    q, s = R.quantize_per_channel(w.numpy())
    mod = sbq.Int8Linear(w, None)
    mod.out_dtype = torch.float16
    y = _np(mod(x.cuda()))
    assert np.isfinite(y).all()
    rows = sorted({r for t in range(0, m, 256) for r in (t, t + 1, t + 127, t + 128, t + 254, t + 255)})
    rng = np.random.default_rng(52)
    rows = np.array(sorted(set(rows) | set(rng.choice(m, 32, replace=False).tolist())))
    xf = x.float().numpy()
    assert R.rel_l2(y[rows], R.int8_linear(xf[rows], q, s)) < REL_L2
    for t in range(0, m, 256):  # tile by tile, so one bad tile cannot hide in the average
        sel = rows[(rows >= t) & (rows < t + 256)]
        assert R.rel_l2(y[sel], R.int8_linear(xf[sel], q, s)) < REL_L2, "M tile %d" % (t // 256)
    _linearity_checks(xf, y, q, s)


# ---- configuration 4: the 36-layer stack's data flow at full width ---------------------------

def _oracle_stack(stack, x: np.ndarray, gate_rounded: bool):
    """The stack (see spikingbrain-cpu_b200/stack.py) with the device path's fp16 rounding points.

    ``gate_rounded``: above 16 rows the gate projection is written to h in fp16 before the up
    GEMM's epilogue forms silu(gate) * up (the decode GEMV keeps it in fp32).
    """
    hd = stack.hidden

    def lin(mod, inp):
        return R.int8_linear(np.asarray(inp, np.float32), mod.qweight.cpu().numpy(), mod.scale.cpu().numpy())

    xf = x.astype(np.float16)
    side = None
    for layer in stack.layers:
        qkvd = lin(layer.qkvd, xf).astype(np.float16)
        g = lin(layer.mlp.gate_proj, xf)
        if gate_rounded:
            g = g.astype(np.float16).astype(np.float64)
        u = lin(layer.mlp.up_proj, xf)
        h = (R.silu(g) * u).astype(np.float16)
        side = np.concatenate([lin(layer.mlp.down_proj, h), lin(layer.dout, qkvd[:, 3 * hd:])], 1).astype(np.float16)
        xf = lin(layer.o, qkvd[:, 2 * hd:3 * hd]).astype(np.float16)
    return xf.astype(np.float32), side.astype(np.float32)


@pytest.fixture(scope="module")
def full_width_stack(sbq):
    # hidden 4096, intermediate 12288 (configuration 4's layer), two layers
    return sbq.stack.ProjectionStack(layers=2, seed=4)


@pytest.mark.parametrize("m", [1, 8, 24, 64, 300])
def test_config4_full_width_stack_vs_oracle(sbq, full_width_stack, m):
    # decode batch 1 and 8 (grouped GEMV launches), 24 and 64 (small-batch GEMM), prefill of 300 tokens
    # (256-token GEMM tiles, a partial last tile)
    stack = full_width_stack
    x = sbq.workloads.activation(m, stack.hidden, seed=400 + m, device="cuda")
    y = _np(stack(x))
    side = _np(stack.side)
    want, want_side = _oracle_stack(stack, x.float().cpu().numpy(), gate_rounded=m > 16)
    assert np.isfinite(want).all()
    assert R.rel_l2(y, want) < REL_L2
    assert R.rel_l2(side, want_side) < REL_L2


def test_config4_prefill_8192_sampled_rows(sbq, full_width_stack):
    # the bench's prefill size: every row goes through the device path, the oracle recomputes 40
    # rows (rows are independent through the stack), and the output must be finite everywhere
    stack = full_width_stack
    m = 8192
    x = sbq.workloads.activation(m, stack.hidden, seed=408, device="cuda")
    y = _np(stack(x))
    side = _np(stack.side)
    assert np.isfinite(y).all() and np.isfinite(side).all()
    rng = np.random.default_rng(409)
    rows = np.array(sorted(set([0, 1, 255, 256, 4095, 4096, 8190, 8191]) | set(rng.choice(m, 32, replace=False).tolist())))
    want, want_side = _oracle_stack(stack, x.float().cpu().numpy()[rows], gate_rounded=True)
    assert R.rel_l2(y[rows], want) < REL_L2
    assert R.rel_l2(side[rows], want_side) < REL_L2


# Configuration 4 sharded over 4 and 8 GPUs gives every rank narrow projections: q|k|v|delta_in as
# one [4 * 4096 / g, 4096] shard, o and delta_out [4096 / g, 4096], gate/up [12288 / g, 4096] (the
# fused epilogue) and down [4096 / g, 12288].  One GPU runs them at the decode batches and the
# prefill size, so the kernels' tile, split-K and CTA-pair choices at these widths are checked
# against the oracle without a multi-GPU box (rows covering every M tile at m = 8192).
@pytest.mark.parametrize("world", [4, 8])
@pytest.mark.parametrize("m", [1, 8, 64, 8192])
def test_config4_rank_shard_shapes(sbq, world, m):
    hd, it = 4096, 12288
    rows = np.unique(np.concatenate([np.arange(0, m, 256), np.arange(255, m, 256), [m - 1]])) if m > 64 \
        else np.arange(m)
    xs = {k: sbq.workloads.activation(m, k, seed=k + m + world) for k in (hd, it)}
    for n, k in ((4 * hd // world, hd), (hd // world, hd), (hd // world, it)):
        w = sbq.workloads.float_weight(n, k, seed=n + k + world)
        q, s = R.quantize_per_channel(w.numpy())
        y = sbq.Int8Linear(w, None)(xs[k].cuda())
        want = R.int8_linear(xs[k].float().numpy()[rows], q, s)
        assert R.rel_l2(_np(y)[rows], want) < REL_L2, (n, k)
    n = it // world
    g = sbq.workloads.float_weight(n, hd, seed=world + 6)
    u = sbq.workloads.float_weight(n, hd, seed=world + 7)
    d = sbq.workloads.float_weight(hd, it, seed=world + 8)
    mlp = sbq.FusedGatedMLP(sbq.Int8Linear(g, None), sbq.Int8Linear(u, None), sbq.Int8Linear(d, None), shards=world)
    h = mlp.gateup_into(xs[hd].cuda(), torch.empty(m, n, dtype=torch.float16, device="cuda"))
    x_rows = xs[hd].float().numpy()[rows]
    want = R.silu(R.int8_linear(x_rows, *R.quantize_per_channel(g.numpy()))) * \
        R.int8_linear(x_rows, *R.quantize_per_channel(u.numpy()))
    assert R.rel_l2(_np(h)[rows], want) < REL_L2
    assert sbq._lib.load().sbq_check_device_error() == 0
