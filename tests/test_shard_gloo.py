"""Host-side logic of the output-channel sharding, run as two gloo ranks on the CPU.

Checks that the all-gather + reorder used between sharded projections reassembles exactly the
unsharded activation, for decode (one row) and prefill (many rows) shapes, and that every rank
takes its row range of the weight the way the stack does.
"""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    import importlib
    import sys

    sys.path.insert(0, str(ROOT))
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        stack_mod = importlib.import_module("spikingbrain-cpu_b200.stack")

        class Stub:
            pass

        stub = Stub()
        stub.world, stub.group = world, dist.group.WORLD
        out = {}
        for m in (1, 5):
            full = torch.arange(m * 64, dtype=torch.float32).reshape(m, 64)
            part = full[:, rank * 64 // world:(rank + 1) * 64 // world]
            got = stack_mod.ProjectionStack._gather(stub, part)
            out[m] = bool(torch.equal(got, full))
            # the side outputs: each rank holds [down slice | delta_out slice] in one buffer; the
            # gathered blocks reorder to [down | delta_out] in channel order
            hd = 32
            down, dout = full[:, :hd], full[:, hd:] + 1000.0
            s = hd // world
            od = torch.cat([down[:, rank * s:(rank + 1) * s], dout[:, rank * s:(rank + 1) * s]], 1)
            side = stack_mod.side_layout(stack_mod.ProjectionStack._gather(stub, od), world, hd)
            out["side%d" % m] = bool(torch.equal(side, torch.cat([down, dout], 1)))
        results[rank] = out
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_gather_reassembles_sharded_output(world):
    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    results = mgr.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    for r in range(world):
        assert results[r] == {1: True, 5: True, "side1": True, "side5": True}
