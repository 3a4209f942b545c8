"""Shared-input projection groups (model.py:317-333, :363-365): the projections of a hybrid block that
read the same x, run as one launch over their concatenated weights, against separate calls.

int8: each member's output within the format's tolerance of its own Int8Linear call and of the
oracle (2e-5 relative L2 for fp32 x, 1e-3 otherwise).  int8-dyn: bit-identical to separate
DynamicInt8Linear calls (the per-tensor quantisation depends on x alone).
"""

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import quant_ref as R

pytestmark = pytest.mark.gpu

HID = 2560
# (name, out_features) of the hybrid block's projections that read x (checkpoint sizes)
SHAPES = [("sse_q_proj", 4096), ("sse_k_proj", 4096), ("sse_v_proj", 4096), ("lora_q_proj.0", 128),
          ("lora_k_proj.0", 128), ("sse_a_proj", 64), ("sse_b_proj", 64), ("sse_e_proj", 4), ("swa_q_proj", 4096),
          ("swa_k_proj", 1024), ("swa_v_proj", 1024)]


def _block(sbq, fmt, seed):
    """A module with the hybrid block's attribute layout, every projection in format fmt."""
    blk = nn.Module()
    weights = {}
    for i, (name, n) in enumerate(SHAPES):
        w = sbq.workloads.float_weight(n, HID, seed=seed + i)
        weights[name] = w
        mod = sbq.make_linear(fmt, w)
        if "." in name:
            head, _ = name.split(".")
            if not hasattr(blk, head):
                setattr(blk, head, nn.Sequential(mod, sbq.make_linear(fmt, sbq.workloads.float_weight(4096, 128, seed=seed + 50 + i))))
            else:
                getattr(blk, head)[0] = mod
        else:
            setattr(blk, name, mod)
    return blk, weights


def _outputs(blk, x):
    return [blk.get_submodule(name)(x) for name, _ in SHAPES]


@pytest.mark.parametrize("m,xdtype", [(1, torch.float32), (7, torch.float32), (512, torch.float32),
                                      (300, torch.float16), (1, torch.bfloat16)])
def test_int8_group_matches_separate_calls(sbq, m, xdtype):
    blk, weights = _block(sbq, "int8", 900)
    x = sbq.workloads.activation(m, HID, seed=m, dtype=xdtype).cuda()
    want = _outputs(blk, x)
    group = sbq.groups.fuse_shared_inputs(blk, sbq.groups.HYBRID_SHARED_INPUTS)
    assert group.n_pad == sum((n + 15) // 16 * 16 for _, n in SHAPES)
    got = _outputs(blk, x)
    tol = 2e-5 if xdtype == torch.float32 else 1e-3
    xf = x.float().cpu().numpy()
    for (name, n), g, w in zip(SHAPES, got, want):
        assert tuple(g.shape) == (m, n), name
        assert R.rel_l2(g.cpu().numpy(), w.cpu().numpy()) < tol, name
        q, s = R.quantize_per_channel(weights[name].numpy())
        assert R.rel_l2(g.cpu().numpy(), R.int8_linear(xf, q, s)) < tol, name
    # the lora pair still runs through its second stage on the group's slice
    t = blk.lora_q_proj(x)
    assert tuple(t.shape) == (m, 4096) and torch.isfinite(t).all()


@pytest.mark.parametrize("m", [1, 64, 512])
def test_dyn_group_bit_identical(sbq, m):
    blk, _ = _block(sbq, "int8-dyn", 950)
    x = sbq.workloads.activation(m, HID, seed=m + 1, dtype=torch.float32).cuda()
    want = _outputs(blk, x)
    sbq.groups.fuse_shared_inputs(blk, sbq.groups.HYBRID_SHARED_INPUTS)
    got = _outputs(blk, x)
    for (name, _), g, w in zip(SHAPES, got, want):
        assert torch.equal(g, w), name


def test_group_host_tensors_and_recompute(sbq):
    blk, _ = _block(sbq, "int8", 990)
    x = sbq.workloads.activation(3, HID, seed=5, dtype=torch.float32)
    want = [o.clone() for o in _outputs(blk, x)]
    group = sbq.groups.fuse_shared_inputs(blk, sbq.groups.HYBRID_SHARED_INPUTS)
    got = _outputs(blk, x)
    assert all(g.device.type == "cpu" for g in got)
    for g, w in zip(got, want):
        assert R.rel_l2(g.numpy(), w.numpy()) < 2e-5
    # a member called twice with the same x recomputes; a new x gives new results
    again = blk.sse_q_proj(x)
    assert torch.equal(again, got[0])
    x2 = x * 2.0
    assert R.rel_l2(blk.sse_q_proj(x2).numpy(), 2.0 * got[0].numpy()) < 2e-5
    assert len(group.sizes) == len(SHAPES)
