"""Decode GEMV launches on several streams at once.

The GEMV's work counters and split-K scratch live in device arrays of the library, divided into
per-stream lanes (include/sbq.h, "Streams and host threads").  Split-K launches - few output tiles
and a long K, as in the real model's N = 4 / 64 projections and every sharded step - run here on
two streams at the same time and must give, bit for bit, what each gives alone.
"""

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _plan_parts(sbq, n, k, m, nmat=1):
    L = sbq._lib
    shapes = (ctypes.c_int64 * 3)(n, k, nmat)
    parts = (ctypes.c_int * 1)()
    sm = torch.cuda.get_device_properties(0).multi_processor_count
    L.call("sbq_gemv_plan_parts", shapes, 1, 3 * sm, m, parts)
    return parts[0]


@pytest.mark.parametrize("m", [1, 4])
def test_split_k_launches_on_two_streams(sbq, m):
    shapes = [(64, 12288), (96, 9728)]
    assert all(_plan_parts(sbq, n, k, m) > 1 for n, k in shapes), "the shapes must take split-K units"
    mods = [sbq.Int8Linear(sbq.workloads.float_weight(n, k, seed=500 + i), torch.randn(n)) for i, (n, k) in enumerate(shapes)]
    xs = [sbq.workloads.activation(m, k, seed=510 + i).cuda() for i, (_, k) in enumerate(shapes)]
    want = [mod(x) for mod, x in zip(mods, xs)]
    torch.cuda.synchronize()
    reps = 40
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    outs = [[torch.empty(m, mod.out_features, device="cuda") for _ in range(reps)] for mod in mods]
    for s in streams:
        s.wait_stream(torch.cuda.current_stream())
    for r in range(reps):  # issue alternately so the two streams' launches overlap on the GPU
        for j, s in enumerate(streams):
            with torch.cuda.stream(s):
                mods[j].forward_into(xs[j], outs[j][r])
    torch.cuda.synchronize()
    for j in range(2):
        for r in range(reps):
            assert torch.equal(outs[j][r], want[j]), "stream %d, launch %d" % (j, r)
    assert sbq._lib.load().sbq_check_device_error() == 0
