"""The fused rank-128 LoRA pair (model.py:287-288: lora_q_proj / lora_k_proj = Linear(2560 -> 128) then
Linear(128 -> 4096), both int8) against the oracle and against the two projections called in turn.

Tolerance: the intermediate stays fp32 (the second stage reads it split into bf16 high + low parts),
so the pair matches the float64 oracle within 1e-4 relative L2 for fp32 x (the reference's type) and
1e-3 for 16-bit x.
"""

import numpy as np
import pytest
import torch
import torch.nn as nn

from oracle import quant_ref as R

pytestmark = pytest.mark.gpu


def _pair(sbq, r=128, k=2560, n=4096, seed=77):
    a = sbq.workloads.float_weight(r, k, seed=seed)
    b = sbq.workloads.float_weight(n, r, seed=seed + 1)
    return a, b, sbq.Int8Linear(a, None), sbq.Int8Linear(b, None)


@pytest.mark.parametrize("m", [1, 3, 8, 9, 16])
@pytest.mark.parametrize("xdtype", [torch.float32, torch.float16, torch.bfloat16])
def test_fused_pair_vs_oracle(sbq, m, xdtype):
    a, b, la, lb = _pair(sbq)
    fused = sbq.FusedLoRAPair(la, lb)
    x = sbq.workloads.activation(m, 2560, seed=m + 5, dtype=xdtype)
    y = fused(x.cuda())
    assert y.dtype == torch.float32 and tuple(y.shape) == (m, 4096)
    qa, sa = R.quantize_per_channel(a.numpy())
    qb, sb = R.quantize_per_channel(b.numpy())
    want = R.int8_linear(R.int8_linear(x.float().numpy(), qa, sa).astype(np.float32), qb, sb)
    tol = 1e-4 if xdtype == torch.float32 else 1e-3
    assert R.rel_l2(y.cpu().numpy(), want) < tol
    # and the two projections in turn (the reference's Sequential)
    assert R.rel_l2(y.cpu().numpy(), lb(la(x.cuda())).cpu().numpy()) < tol
    assert sbq._lib.load().sbq_check_device_error() == 0


@pytest.mark.parametrize("r,n,k", [(64, 1000, 512), (128, 4096, 2560), (16, 40, 64), (112, 300, 4096)])
def test_fused_pair_shapes(sbq, r, n, k):
    a, b, la, lb = _pair(sbq, r, k, n, seed=r + n)
    fused = sbq.FusedLoRAPair(la, lb)
    fused.out_dtype = torch.float16
    x = sbq.workloads.activation(5, k, seed=k, dtype=torch.float32)
    y = fused(x.cuda())
    assert y.dtype == torch.float16
    qa, sa = R.quantize_per_channel(a.numpy())
    qb, sb = R.quantize_per_channel(b.numpy())
    want = R.int8_linear(R.int8_linear(x.numpy(), qa, sa).astype(np.float32), qb, sb)
    assert R.rel_l2(y.float().cpu().numpy(), want) < 1e-3


def test_fuse_lora_pairs_in_a_module_tree(sbq):
    # prefill sizes fall back to the two projections; host tensors come back on the host
    _, _, la, lb = _pair(sbq, seed=5)
    blk = nn.Module()
    blk.lora_q_proj = nn.Sequential(la, lb)
    want_dec = blk.lora_q_proj(sbq.workloads.activation(1, 2560, seed=1, dtype=torch.float32).cuda())
    x_pre = sbq.workloads.activation(40, 2560, seed=2, dtype=torch.float32)
    want_pre = blk.lora_q_proj(x_pre.cuda())
    assert sbq.fuse_lora_pairs(blk) == 1 and isinstance(blk.lora_q_proj, sbq.FusedLoRAPair)
    got_dec = blk.lora_q_proj(sbq.workloads.activation(1, 2560, seed=1, dtype=torch.float32).cuda())
    assert R.rel_l2(got_dec.cpu().numpy(), want_dec.cpu().numpy()) < 1e-4
    got_pre = blk.lora_q_proj(x_pre)
    assert got_pre.device.type == "cpu"
    assert torch.equal(got_pre, want_pre.cpu())


def test_fused_pair_rejects_unsupported(sbq):
    _, _, la, _ = _pair(sbq, r=128)
    _, _, lc, ld = _pair(sbq, r=144, k=256, n=64, seed=9)
    with pytest.raises(ValueError):
        sbq.FusedLoRAPair(lc, ld)  # inner size above 128
    with pytest.raises(ValueError):
        sbq.FusedLoRAPair(la, ld)  # shapes do not chain
