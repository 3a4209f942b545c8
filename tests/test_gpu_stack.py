"""GPU parity of the synthetic projection stack (configuration 4's data flow) at a reduced size.

The oracle composes the per-projection CPU restatement (quant.py:41-53 and model.py:239-240) with
the same fp16 rounding points as the device path.  Tolerance: relative L2 1e-3 on the final
activation after two layers.
"""

import numpy as np
import pytest
import torch

from oracle import quant_ref as R

pytestmark = pytest.mark.gpu


def _oracle_stack(stack, x):
    hd = stack.hidden

    def lin(mod, inp):
        return R.int8_linear(np.asarray(inp, np.float32), mod.qweight.cpu().numpy(), mod.scale.cpu().numpy())

    xf = x.cpu().numpy().astype(np.float16)
    side = None
    for layer in stack.layers:
        qkvd = lin(layer.qkvd, xf).astype(np.float16)
        g = lin(layer.mlp.gate_proj, xf)
        u = lin(layer.mlp.up_proj, xf)
        h = (R.silu(g) * u).astype(np.float16)
        side = np.concatenate([lin(layer.mlp.down_proj, h), lin(layer.dout, qkvd[:, 3 * hd:])], 1).astype(np.float16)
        xf = lin(layer.o, qkvd[:, 2 * hd:3 * hd]).astype(np.float16)
    return xf, side


@pytest.mark.parametrize("m", [1, 3, 16])
def test_small_stack_vs_oracle(sbq, m):
    stack = sbq.stack.ProjectionStack(layers=2, hidden=256, inter=768, seed=1)
    x = sbq.workloads.activation(m, 256, seed=2, device="cuda")
    y = stack(x)
    assert y.dtype == torch.float16 and tuple(y.shape) == (m, 256)
    want, side = _oracle_stack(stack, x)
    assert np.isfinite(want).all() and np.isfinite(side).all()
    assert R.rel_l2(y.float().cpu().numpy(), want.astype(np.float32)) < 1e-3
    # the last layer's side outputs [down(h) | delta_out(delta_in)]
    assert R.rel_l2(stack.side.float().cpu().numpy(), side.astype(np.float32)) < 1e-3


def test_captured_stack_matches_eager(sbq):
    stack = sbq.stack.ProjectionStack(layers=3, hidden=512, inter=1024, seed=3)
    runner = sbq.stack.CapturedStack(stack, m=1)
    x = sbq.workloads.activation(1, 512, seed=4)
    eager = stack(x.cuda()).cpu()
    host = runner(x).clone()
    assert torch.equal(host, eager)
    dev = runner(x.cuda()).cpu()
    assert torch.equal(dev, eager)
    again = runner.run().cpu()
    assert torch.equal(again, eager)
    runner.release()


@pytest.mark.parametrize("m", [1, 8])
def test_stack_activations_stay_bounded(sbq, m):
    # the benchmark's 36-layer stack at full width: the folded scales keep every output finite and
    # near unit scale to the last layer (the layer chain runs through the linear o(v) path)
    stack = sbq.stack.ProjectionStack(seed=4)
    y = stack(sbq.workloads.activation(m, 4096, seed=5, device="cuda")).float()
    side = stack.side.float()
    assert torch.isfinite(y).all() and torch.isfinite(side).all()
    assert 0.5 < float(y.std()) < 2.0
    assert 0.5 < float(side[:, :4096].std()) < 2.0 and 0.5 < float(side[:, 4096:].std()) < 2.0


@pytest.mark.parametrize("layers,hidden,inter", [(3, 512, 1024), (2, 4096, 12288)])
def test_decode_program_matches_grouped_launches(sbq, layers, hidden, inter):
    # the one-launch decode program computes every tile exactly as the grouped launches do
    stack = sbq.stack.ProjectionStack(layers=layers, hidden=hidden, inter=inter, seed=6)
    x = sbq.workloads.activation(1, hidden, seed=7, device="cuda")
    want = stack(x)
    prog = stack.decode_program(x.clone())
    for _ in range(2):  # the counters are cleared by every run
        got = prog.run()
        torch.cuda.synchronize()
        assert torch.equal(got, want)
    assert sbq._lib.load().sbq_check_device_error() == 0
    # and the captured runner (which uses it) agrees with eager
    runner = sbq.stack.CapturedStack(stack, m=1, use_program=True)
    assert runner.program is not None
    assert torch.equal(runner(x.cpu()).cuda(), want)
    runner.release()


@pytest.mark.parametrize("m", [1, 40])
def test_module_api_path_host_and_device(sbq, m):
    # the same data flow through the drop-in's public module calls only (the reference model's way of
    # calling its projections): host tensors in and out, or device tensors with no host sync
    stack = sbq.stack.ProjectionStack(layers=2, hidden=256, inter=768, seed=11)
    x = sbq.workloads.activation(m, 256, seed=12)
    y_host = stack.forward_modules(x)
    assert y_host.device.type == "cpu" and y_host.dtype == torch.float16
    y_dev = stack.forward_modules(x.cuda())
    assert y_dev.device.type == "cuda"
    assert torch.equal(y_host, y_dev.cpu())
    want, _ = _oracle_stack(stack, x)
    assert R.rel_l2(y_host.float().numpy(), want.astype(np.float32)) < 1e-3


@pytest.mark.parametrize("m", [1, 8, 40])
def test_overlapped_launches_match_plain_grouping(sbq, m):
    # one GPU runs each layer's side outputs as ready jobs of the next launch (decode GEMV, m <= 16)
    # or on a second stream (one GEMM per projection above 16 rows); the results equal the plain
    # grouping bit for bit, eagerly and over repeated CUDA-graph replays (which would expose a
    # launch that reads an input before it is written)
    kw = dict(layers=4, hidden=1024, inter=3072, seed=7)
    ov = sbq.stack.ProjectionStack(**kw)
    plain = sbq.stack.ProjectionStack(overlap=False, **kw)
    assert ov.overlap and not plain.overlap
    assert ov.launches_per_step(m) == plain.launches_per_step(m) + (1 if m <= 16 else 0)
    x = sbq.workloads.activation(m, 1024, seed=8, device="cuda")
    want = plain(x)
    want_side = plain.side.clone()
    assert torch.equal(ov(x), want) and torch.equal(ov.side, want_side)
    runner = sbq.stack.CapturedStack(ov, m=m)
    runner.x.copy_(x)
    for _ in range(20):
        assert torch.equal(runner.run(), want)
    assert torch.equal(ov.side, want_side)
    runner.release()
    assert sbq._lib.load().sbq_check_device_error() == 0
