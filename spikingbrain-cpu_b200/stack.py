"""Synthetic 36-layer projection stack (benchmark configuration 4), optionally output-channel sharded.

Each layer holds the projections the hybrid model runs through its int8 linears
(spikingbrain_cpu/model.py:232-301): q/k/v/o and the delta-net in/out projections
([hidden x hidden] each) and the gate/up/down MLP ([inter x hidden], [hidden x inter]).  The data
flow between them is real, so every projection depends on the one before it:

    qkvd = [q | k | v | delta_in](x)          one GEMV/GEMM over the concatenated weight (fp16 out)
    od   = [o(v) | delta_out(delta_in)]       two launches writing one fp16 buffer
    h    = silu(gate(x)) * up(x)              fused gate/up kernel (fp16 h)
    x'   = down(h)                            fp16, the next layer's input

so a decode step streams every weight of every layer exactly once.  Constant factors are folded
into the per-row scales of the projections whose outputs are consumed (v, delta_in, down) so
the activations stay near unit variance over 36 layers; the int8 weights themselves follow the
reference quantiser on ``N(0, 0.02)`` weights.

Sharding (``world > 1``): rank r owns rows [r n / world, (r+1) n / world) of every projection and
produces that slice of each output; ``torch.distributed.all_gather_into_tensor`` (NCCL over
NVLink) assembles the full activation before its consumer.  x is replicated.
"""

from __future__ import annotations

import ctypes
import math

import torch
import torch.nn as nn

from . import workloads as W
from .mlp import FusedGatedMLP
from .quant import Int8Linear


def _fold(k: int, second_moment: float = 1.0) -> float:
    """Factor that maps sum_k w x (w ~ N(0, 0.02)) of inputs with E[x^2] = second_moment to unit variance."""
    return 1.0 / math.sqrt(k * 0.02 * 0.02 * second_moment)


def _h_moment(hidden: int) -> float:
    """E[(silu(g) * u)^2] for independent g, u ~ N(0, 0.02^2 * hidden) (unit-variance x), by quadrature."""
    var = hidden * 0.02 * 0.02
    sd = math.sqrt(var)
    t = torch.linspace(-10.0, 10.0, 4001, dtype=torch.float64) * sd
    pdf = torch.exp(-0.5 * (t / sd) ** 2) / (sd * math.sqrt(2.0 * math.pi))
    silu2 = (t * torch.sigmoid(t)) ** 2
    return float((silu2 * pdf).sum() * (t[1] - t[0])) * var


class StackLayer(nn.Module):
    def __init__(self, layer: int, hidden: int, inter: int, seed: int, device, rank: int = 0, world: int = 1):
        super().__init__()
        self.hidden, self.inter, self.rank, self.world = hidden, inter, rank, world
        dev = torch.device(device)
        base = seed * 1000 + layer * 16

        def rows(w: torch.Tensor) -> torch.Tensor:
            n = w.shape[0]
            return w[rank * n // world:(rank + 1) * n // world]

        def shard(n: int, k: int, idx: int) -> torch.Tensor:
            return rows(W.float_weight(n, k, seed=base + idx, device=dev))

        f_h = _fold(hidden)
        # the concatenation is sharded as one matrix so the gathered output keeps the q|k|v|d order
        qkvd_w = rows(torch.cat([W.float_weight(hidden, hidden, seed=base + i, device=dev) for i in range(4)], 0))
        self.qkvd = Int8Linear(qkvd_w, None, device=dev)
        self.qkvd.scale.mul_(f_h)
        self.qkvd.out_dtype = torch.float16
        self.o = Int8Linear(shard(hidden, hidden, 4), None, device=dev)
        self.o.scale.mul_(f_h)
        self.o.out_dtype = torch.float16
        self.dout = Int8Linear(shard(hidden, hidden, 5), None, device=dev)
        self.dout.scale.mul_(f_h)
        self.dout.out_dtype = torch.float16
        gate = Int8Linear(shard(inter, hidden, 6), None, device=dev)
        up = Int8Linear(shard(inter, hidden, 7), None, device=dev)
        down = Int8Linear(shard(hidden, inter, 8), None, device=dev)
        down.scale.mul_(_fold(inter, _h_moment(hidden)))
        down.out_dtype = torch.float16
        self.mlp = FusedGatedMLP(gate, up, down, shards=world)
        del qkvd_w

    def weight_bytes(self) -> int:
        mods = (self.qkvd, self.o, self.dout, self.mlp.gate_proj, self.mlp.up_proj, self.mlp.down_proj)
        return sum(m.out_features * m.in_features for m in mods)


class ProjectionStack(nn.Module):
    """The stack; ``forward(x)`` maps fp16 [m, hidden] to fp16 [m, hidden] on the device."""

    def __init__(self, layers: int = W.LAYERS, hidden: int = W.HIDDEN, inter: int = W.INTER, seed: int = 4,
                 device=None, group=None):
        super().__init__()
        import torch.distributed as dist

        self.group = group
        self.world = dist.get_world_size(group) if group is not None else 1
        self.rank = dist.get_rank(group) if group is not None else 0
        for n in (hidden, inter):
            if n % (16 * self.world):
                raise ValueError("%d rows do not split into %d 16-row shards" % (n, self.world))
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.device, self.hidden, self.inter = dev, hidden, inter
        self.layers = nn.ModuleList(StackLayer(i, hidden, inter, seed, dev, self.rank, self.world)
                                    for i in range(layers))

    def weight_bytes(self) -> int:
        """int8 weight bytes this rank streams per decode step."""
        return sum(layer.weight_bytes() for layer in self.layers)

    def _gather(self, part: torch.Tensor) -> torch.Tensor:
        """[m, n/world] slice on every rank -> [m, n] everywhere (NCCL all-gather + reorder)."""
        if self.world == 1:
            return part
        import torch.distributed as dist

        m, ns = part.shape
        buf = torch.empty(self.world * m, ns, dtype=part.dtype, device=part.device)
        dist.all_gather_into_tensor(buf, part.contiguous(), group=self.group)
        if m == 1:
            return buf.view(1, self.world * ns)
        return buf.view(self.world, m, ns).permute(1, 0, 2).reshape(m, self.world * ns)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """fp16 [m, hidden] on the device -> fp16 [m, hidden] (the last layer's down projection).

        Decode sizes (m <= 16) run each layer as two grouped launches: [gate/up, q|k|v|delta_in]
        (both read x) and [down, o, delta_out] (after their inputs are gathered).
        """
        if x.shape[0] <= 16:
            return self._forward_grouped(x)
        hd, w = self.hidden, self.world
        m = x.shape[0]
        for layer in self.layers:
            qkvd = self._gather(layer.qkvd.forward_into(x, x.new_empty(m, 4 * hd // w)))
            od = x.new_empty(m, 2 * hd // w)
            layer.o.forward_into(qkvd[:, 2 * hd:3 * hd], od[:, :hd // w])
            layer.dout.forward_into(qkvd[:, 3 * hd:], od[:, hd // w:])
            self._gather(od)
            h = self._gather(layer.mlp.gateup_into(x, x.new_empty(m, self.inter // w)))
            x = self._gather(layer.mlp.down_proj.forward_into(h, x.new_empty(m, hd // w)))
        return x

    def _forward_grouped(self, x: torch.Tensor) -> torch.Tensor:
        from .quant import gemv_group

        hd, w = self.hidden, self.world
        m = x.shape[0]
        for layer in self.layers:
            qkvd = x.new_empty(m, 4 * hd // w)
            h = x.new_empty(m, self.inter // w)
            gemv_group([layer.mlp.gateup_job(x, h), layer.qkvd.gemv_job(x, qkvd)], x.dtype, m, x.device)
            qkvd, h = self._gather(qkvd), self._gather(h)
            od = x.new_empty(m, 2 * hd // w)
            xn = x.new_empty(m, hd // w)
            gemv_group([layer.mlp.down_proj.gemv_job(h, xn), layer.o.gemv_job(qkvd[:, 2 * hd:3 * hd], od[:, :hd // w]),
                        layer.dout.gemv_job(qkvd[:, 3 * hd:], od[:, hd // w:])], x.dtype, m, x.device)
            self._gather(od)
            x = self._gather(xn)
        return x

    def decode_program(self, x: torch.Tensor) -> "DecodeProgram":
        """The whole batch-1 decode step as one persistent launch reading ``x`` (see DecodeProgram)."""
        return DecodeProgram(self, x)

    def launches_per_step(self, m: int, program: bool = False) -> int:
        """Kernels of this library one forward launches (one decode program, else grouped launches
        for m <= 16, else one launch per projection)."""
        if program:
            return 1
        if m <= 16:
            return len(self.layers) * 2
        return len(self.layers) * 5


class DecodeProgram:
    """A single-GPU batch-1 decode step of the stack as one launch of the decode program kernel.

    Two stages per layer: [gate/up, q|k|v|delta_in] read the layer input, [down, o, delta_out] read
    their outputs; a grid-wide barrier inside the kernel separates them and the weight stream never
    pauses.  Every layer gets its own activation buffers (written once per step).  ``run()`` reads
    the fixed input buffer ``x`` and returns the fixed output buffer (the last layer's down output).
    """

    def __init__(self, stack: ProjectionStack, x: torch.Tensor):
        from . import _lib as L
        from .quant import _DTYPE_CODE

        if stack.world != 1:
            raise ValueError("the decode program runs on one GPU (no gathers inside a launch)")
        if x.shape != (1, stack.hidden) or x.dtype != torch.float16 or not x.is_contiguous():
            raise ValueError("the decode program takes a contiguous fp16 [1, hidden] input")
        hd, dev = stack.hidden, x.device
        self.stack, self.x = stack, x
        self.buffers = []
        jobs, stage = [], []
        cur = x
        for i, layer in enumerate(stack.layers):
            qkvd = torch.empty(1, 4 * hd, dtype=torch.float16, device=dev)
            h = torch.empty(1, stack.inter, dtype=torch.float16, device=dev)
            od = torch.empty(1, 2 * hd, dtype=torch.float16, device=dev)
            nxt = torch.empty(1, hd, dtype=torch.float16, device=dev)
            self.buffers += [qkvd, h, od, nxt]
            jobs += [layer.mlp.gateup_job(cur, h), layer.qkvd.gemv_job(cur, qkvd)]
            stage += [2 * i, 2 * i]
            jobs += [layer.mlp.down_proj.gemv_job(h, nxt), layer.o.gemv_job(qkvd[:, 2 * hd:3 * hd], od[:, :hd]),
                     layer.dout.gemv_job(qkvd[:, 3 * hd:], od[:, hd:])]
            stage += [2 * i + 1] * 3
            cur = nxt
        self.y = cur
        self.nstages = 2 * len(stack.layers)
        lib = L.load()
        nbytes = int(lib.sbq_gemv_program_bytes(self.nstages))
        self.program = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        self.counters = torch.zeros(self.nstages, dtype=torch.int32, device=dev)
        arr = (L.GemvJob * len(jobs))(*jobs)
        st = (ctypes.c_int * len(stage))(*stage)
        self._code = _DTYPE_CODE[torch.float16]
        L.call("sbq_gemv_program_build", arr, st, len(jobs), self._code, 1, ctypes.c_void_p(self.program.data_ptr()),
               nbytes)

    def run(self) -> torch.Tensor:
        from . import _lib as L
        from .quant import _stream

        L.call("sbq_gemv_program_run", ctypes.c_void_p(self.program.data_ptr()), self.nstages, self._code,
               ctypes.c_void_p(self.counters.data_ptr()), _stream(self.x.device))
        return self.y


class CapturedStack:
    """ProjectionStack.forward captured once in a CUDA graph at a fixed batch size.

    ``run()`` replays it on the device-resident input buffer ``x``; calling the object with a host
    tensor copies it in (from pinned memory), replays the graph, copies the result back into a
    pinned host buffer and waits for it, which is what a host-side caller of a decode step sees.
    Launch overhead of the per-projection kernels disappears inside the graph.
    """

    def __init__(self, stack: ProjectionStack, m: int = 1, stream: torch.cuda.Stream | None = None,
                 use_program: bool = False):
        self.stack = stack
        self.stream = stream or torch.cuda.Stream(stack.device)
        self.x = torch.zeros(m, stack.hidden, dtype=torch.float16, device=stack.device)
        # grouped launches by default; use_program=True runs a batch-1 single-GPU step as one
        # decode-program launch (bit-identical; measured slower than the grouped launches so far)
        self.program = stack.decode_program(self.x) if (m == 1 and stack.world == 1 and use_program) else None
        step = self.program.run if self.program is not None else (lambda: stack(self.x))
        with torch.cuda.stream(self.stream):
            step()  # warm-up outside the capture (allocator, communicators)
        self.stream.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=self.stream):
            self.y = step()
        self.x_host = torch.empty(m, stack.hidden, dtype=torch.float16).pin_memory()
        self.y_host = torch.empty(m, stack.hidden, dtype=torch.float16).pin_memory()

    def run(self) -> torch.Tensor:
        """Replay on the device-resident ``x``; the caller's current stream is ordered after it."""
        caller = torch.cuda.current_stream(self.stack.device)
        self.stream.wait_stream(caller)
        with torch.cuda.stream(self.stream):
            self.graph.replay()
        caller.wait_stream(self.stream)
        return self.y

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        if x.device.type == "cuda":
            # the graph runs on its own (non-blocking) stream: order it after the producer of x and
            # the caller's later work after it
            caller = torch.cuda.current_stream(self.stack.device)
            self.stream.wait_stream(caller)
            with torch.cuda.stream(self.stream):
                self.x.copy_(x)
                self.graph.replay()
            caller.wait_stream(self.stream)
            return self.y
        if x.data_ptr() != self.x_host.data_ptr():
            self.x_host.copy_(x)
        with torch.cuda.stream(self.stream):
            self.x.copy_(self.x_host, non_blocking=True)
            self.graph.replay()
            self.y_host.copy_(self.y, non_blocking=True)
        self.stream.synchronize()
        return self.y_host

    def release(self) -> None:
        """Drop the graph (required before destroying a process group whose NCCL calls it holds)."""
        self.graph.reset()
        self.graph = None
