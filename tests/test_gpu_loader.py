"""GPU parity of the streaming loader repack (the loader's int8 path, spikingbrain_cpu/loader.py:46-51,
:74-88, with quant.py:25-29 / :57-61 on the device).

Weights handed to ``StreamingPacker.make_linear`` in the loader's order must come out exactly as
``make_linear`` builds them - the same int8 values and scales as the reference's quantiser, bit for
bit - including weights larger than a staging buffer (row blocks) and rows that are not a multiple
of 16 or 64 wide.
"""

import numpy as np
import pytest
import torch

from oracle import quant_ref as R

pytestmark = pytest.mark.gpu

SHAPES = [(9728, 2560), (128, 2560), (4, 2560), (4096, 128), (300, 77), (2560, 9728), (64, 2560), (33, 1000)]


@pytest.mark.parametrize("fmt", ["int8", "int8-dyn"])
def test_streaming_packer_matches_reference_quantiser(sbq, fmt):
    packer = sbq.loader.StreamingPacker(staging_bytes=1 << 20)  # 1 MiB: the large weights go in row blocks
    weights = []
    for i, (n, k) in enumerate(SHAPES):
        w = sbq.workloads.float_weight(n, k, seed=700 + i)
        weights.append(w.to(torch.bfloat16) if i % 2 == 0 else w)
    mods = [packer.make_linear(fmt, w) for w in weights]
    packer.finish()
    for w, mod in zip(weights, mods):
        q, s = R.quantize_per_channel(w.float().numpy())
        assert np.array_equal(mod.qweight.cpu().numpy(), q)
        assert np.array_equal(mod.scale.cpu().numpy().view(np.uint32), s.view(np.uint32))
        eager = sbq.make_linear(fmt, w)
        assert torch.equal(mod.packed, eager.packed)
        if fmt == "int8-dyn":
            assert torch.equal(mod.rowsum, eager.rowsum)
            assert isinstance(mod, sbq.DynamicInt8Linear)
        else:
            assert isinstance(mod, sbq.Int8Linear)
    # the modules work straight away (stream-ordered after the packing)
    x = sbq.workloads.activation(3, 2560, seed=9, dtype=torch.float32).cuda()
    y = mods[1](x).cpu().numpy()
    q, s = R.quantize_per_channel(weights[1].float().numpy())
    if fmt == "int8":
        assert R.rel_l2(y, R.int8_linear(x.cpu().numpy(), q, s)) < 2e-5
    else:
        assert np.array_equal(y.view(np.uint32), R.dyn_linear(x.cpu().numpy(), q, s)[0].view(np.uint32))


def test_streaming_packer_host_tensor_reusable_after_call(sbq):
    # the loader frees each shard's tensors right after make_linear returns (loader.py:87): the
    # packer must have taken its copy by then
    packer = sbq.loader.StreamingPacker(staging_bytes=1 << 20)
    buf = sbq.workloads.float_weight(512, 1024, seed=1)
    want = [R.quantize_per_channel(buf.numpy())]
    a = packer.make_linear("int8", buf)
    buf.mul_(-3.0)  # overwrite the host tensor at once
    want.append(R.quantize_per_channel(buf.numpy()))
    b = packer.make_linear("int8", buf)
    packer.finish()
    assert np.array_equal(a.qweight.cpu().numpy(), want[0][0])
    assert np.array_equal(b.qweight.cpu().numpy(), want[1][0])


def test_streaming_packer_formats_and_errors(sbq):
    packer = sbq.loader.StreamingPacker(staging_bytes=1 << 20)
    f = packer.make_linear("float32", torch.randn(8, 16))
    assert isinstance(f, sbq.FloatLinear)
    with pytest.raises(ValueError, match="unknown weight format"):
        packer.make_linear("int4", torch.randn(8, 16))
    with pytest.raises(ValueError):
        packer.make_linear("int8", torch.randn(8, 16, 2))
    with pytest.raises(ValueError, match="staging"):
        packer.make_linear("int8", torch.randn(16, 20000))  # 16 rows of fp32 exceed 1 MiB
    packer.finish()
