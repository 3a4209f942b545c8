"""One rank of the sharded-stack parity check (run by tests/test_gpu_multi.py under torchrun).

Every rank builds the unsharded stack on its own GPU as the reference (the seeded weights are the
same on every rank), then the output-channel sharded stack with each exchange ("peer": GEMV outputs
stored to every rank over NVLink; "nccl": all-gather), and checks that every sharded result is
bit-identical to the unsharded one: eager decode (m = 1, 3, 16), the captured decode step replayed
back to back on 24 inputs and called with device and host inputs, and the decode program.  An
m = 80 prefill (NCCL gathers) is checked against the int8 format's 1e-3 relative L2 instead: the
sharded GEMMs split K differently.  Exits non-zero on any mismatch.
"""

from __future__ import annotations

import datetime
import importlib
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch
import torch.distributed as dist


def main() -> int:
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    sbq = importlib.import_module("spikingbrain-cpu_b200")
    dev = torch.device("cuda", local)
    shape = dict(layers=3, hidden=1024, inter=2048, seed=11, device=dev)
    ref = sbq.stack.ProjectionStack(**shape)
    failures = []

    def check(name, got, want):
        if not torch.equal(got.cpu(), want.cpu()):
            d = (got.float() - want.float()).abs().max().item()
            failures.append("%s: max |diff| %g" % (name, d))

    def check_close(name, got, want, rel=1e-3):
        # prefill GEMMs split K by the shape of each rank's slice (fewer tiles per rank, more K parts),
        # so sharded and unsharded sums are rounded differently: compare with the format's tolerance
        g, w = got.float().cpu(), want.float().cpu()
        err = ((g - w).norm() / w.norm()).item()
        if not err < rel:
            failures.append("%s: relative L2 %g" % (name, err))

    # "peer" runs each layer's side outputs as ready jobs of the next layer's first launch by default
    # ("peer-plain": the two-launches-per-layer grouping)
    for exchange in ("peer", "peer-plain", "nccl"):
        st = sbq.stack.ProjectionStack(group=dist.group.WORLD, exchange=exchange.split("-")[0],
                                       overlap=exchange != "peer-plain", **shape)
        if st.overlap != (exchange == "peer"):
            failures.append("%s: overlap %s" % (exchange, st.overlap))
        for m in (1, 3, 16):
            x = sbq.workloads.activation(m, shape["hidden"], seed=20 + m, device=dev)
            check("%s eager m=%d" % (exchange, m), st(x).clone(), ref(x))
            check("%s eager side outputs m=%d" % (exchange, m), st.side.clone(), ref.side)
        x = sbq.workloads.activation(80, shape["hidden"], seed=3, device=dev)
        check_close("%s prefill m=80" % exchange, st(x).clone(), ref(x))
        check_close("%s prefill side outputs m=80" % exchange, st.side.clone(), ref.side)
        run = sbq.stack.CapturedStack(st, m=1)
        # back-to-back replays with a new input each: a stale slice from an earlier step would show
        xs = [sbq.workloads.activation(1, shape["hidden"], seed=100 + i, device=dev) for i in range(24)]
        outs = []
        for x in xs:
            run.x.copy_(x)
            outs.append(run.run().clone())
        for i, (x, y) in enumerate(zip(xs, outs)):
            check("%s back-to-back replay %d" % (exchange, i), y, ref(x))
        for i in range(4):
            x = sbq.workloads.activation(1, shape["hidden"], seed=40 + i, device=dev)
            check("%s graph replay %d" % (exchange, i), run(x).clone(), ref(x))
            xh = x.cpu()
            check("%s graph host call %d" % (exchange, i), run(xh).clone(), ref(x))
        if exchange == "peer":
            # the whole sharded step as one decode-program launch per rank
            prog = sbq.stack.CapturedStack(st, m=1, use_program=True)
            assert prog.program is not None
            for i in range(12):
                x = sbq.workloads.activation(1, shape["hidden"], seed=200 + i, device=dev)
                check("peer program replay %d" % i, prog(x).clone(), ref(x))
            prog.release()
        torch.cuda.synchronize()
        status = sbq._lib.load().sbq_check_device_error()
        if status:
            failures.append("%s: device error %d" % (exchange, status))
        run.release()
        dist.barrier()
        if st.peer is not None:
            st.peer.close()
    dist.barrier()
    dist.destroy_process_group()
    for f in failures:
        print("rank %d: %s" % (rank, f), flush=True)
    print("rank %d: %s" % (rank, "ok" if not failures else "FAILED"), flush=True)
    return 1 if failures else 0


if __name__ == "__main__":
    sys.exit(main())
