"""Synthetic 36-layer projection stack (benchmark configuration 4), optionally output-channel sharded.

Each layer holds the projections the hybrid model runs through its int8 linears
(spikingbrain_cpu/model.py:232-301): q/k/v/o and the delta-net in/out projections
([hidden x hidden] each) and the gate/up/down MLP ([inter x hidden], [hidden x inter]).  The data
flow between them is real, so every projection depends on the one before it:

    qkvd = [q | k | v | delta_in](x)          one GEMV/GEMM over the concatenated weight (fp16 out)
    h    = silu(gate(x)) * up(x)              fused gate/up kernel (fp16 h)
    od   = [down(h) | delta_out(delta_in)]    the layer's side outputs, one fp16 buffer
    x'   = o(v)                               fp16, the next layer's input

so a decode step streams every weight of every layer exactly once, and each layer's launches wait
for the previous layer.  Constant factors are folded into the per-row scales (qkvd, o, delta_out,
down) so every output has about unit variance; the int8 weights themselves follow the reference
quantiser on ``N(0, 0.02)`` weights.  The chain from layer to layer runs through the linear
attention path: h is quadratic in x, so a chain through down(h) is unstable under any constant
scale (a layer input slightly below unit scale shrinks quadratically from layer to layer and
reaches zero in fp16 within about twelve layers).  The model's residual stream and norms are not
part of the quantised-linear path.

Sharding (``world > 1``): rank r owns rows [r n / world, (r+1) n / world) of every projection and
produces that slice of each output; x is replicated.  Two ways assemble the full activation before
its consumer:

* ``exchange="peer"`` (decode, m <= 16): every GEMV stores its slice straight into every rank's
  full-width buffer over NVLink and signals a per-launch arrival counter on every rank; the next
  launch waits on its local counter (``PeerExchange``).  Two synchronisation points per layer and
  no collective launches.
* ``exchange="nccl"`` (and every prefill size): ``torch.distributed.all_gather_into_tensor`` after
  each sharded projection.
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


class _DeviceBytes:
    """``__cuda_array_interface__`` of raw device memory, so torch can view it without owning it."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "strides": None, "version": 2}


class PeerExchange:
    """Rank-symmetric arena of a sharded stack's decode activations and arrival counters.

    Every rank allocates the same layout (``libsbq`` peer arena), exports it with a CUDA IPC handle
    and maps every other rank's arena, so that a GEMV can store its output slice into all ranks'
    full-width buffers and signal their counters (``sbq_gemv_w8_group_peer``).  Per layer: the full
    ``qkvd`` [m_max, 4 hidden], ``h`` [m_max, inter], ``od`` [m_max, 2 hidden] and ``x'`` [m_max, hidden]
    buffers (fp16), one signal (32 counter copies) and one count-out word per launch and one wait
    state per waiting launch.
    The ranks must be distinct GPUs of one node with peer access.
    """

    def __init__(self, stack: "ProjectionStack", m_max: int = 16):
        import torch.distributed as dist

        from . import _lib as L

        self.L, self.lib = L, L.load()
        self.stack, self.m_max = stack, m_max
        w, rank, dev = stack.world, stack.rank, stack.device
        if w > L.MAX_PEERS:
            raise ValueError("at most %d ranks share a peer exchange" % L.MAX_PEERS)
        props = torch.cuda.get_device_properties(dev)
        ident = str(getattr(props, "uuid", "")) or "%s:%s" % (getattr(props, "pci_bus_id", ""), dev.index)
        ids = [None] * w
        dist.all_gather_object(ids, ident, group=stack.group)
        if len(set(ids)) != w:
            raise ValueError("peer exchange needs one GPU per rank (ranks share a device)")
        hd, it = stack.hidden, stack.inter
        off = 0

        def take(nbytes: int) -> int:
            nonlocal off
            o = off
            off += (nbytes + 255) // 256 * 256
            return o

        self.buf = []  # per layer: offsets of qkvd, h, od, x'
        for _ in stack.layers:
            self.buf.append([take(m_max * n * 2) for n in (4 * hd, it, 2 * hd, hd)])
        sig = L.PEER_SIGNAL_BYTES
        self.cnt = [[take(sig), take(sig)] for _ in stack.layers]    # signal of launch 1 / 2
        self.done = [[take(128), take(128)] for _ in stack.layers]   # CTA count-out of launch 1 / 2
        self.state = [[take(128), take(128)] for _ in stack.layers]  # wait state of launch 1 / 2
        self.final_state = take(128)
        self.cnt_last, self.done_last, self.state_last = take(sig), take(128), take(128)  # side-output launch
        self.nstages = 2 * len(stack.layers)
        self.prog_sync = take(int(self.lib.sbq_gemv_program_sync_bytes(self.nstages)))  # sharded decode program
        self.nbytes = off
        base = ctypes.c_void_p()
        L.call("sbq_peer_alloc", off, ctypes.byref(base))
        self.base = base.value
        handle = (ctypes.c_uint8 * L.PEER_HANDLE_BYTES)()
        L.call("sbq_peer_handle", ctypes.c_void_p(self.base), handle)
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=dev)
        every = torch.empty(w * L.PEER_HANDLE_BYTES, dtype=torch.uint8, device=dev)
        dist.all_gather_into_tensor(every, mine, group=stack.group)
        every = every.cpu().view(w, L.PEER_HANDLE_BYTES)
        self.peers = []
        for p in range(w):
            if p == rank:
                self.peers.append(self.base)
                continue
            h = (ctypes.c_uint8 * L.PEER_HANDLE_BYTES)(*every[p].tolist())
            ptr = ctypes.c_void_p()
            L.call("sbq_peer_open", h, ctypes.byref(ptr))
            self.peers.append(ptr.value)
        self.arena = torch.as_tensor(_DeviceBytes(self.base, self.nbytes), device=dev)
        dist.barrier(group=stack.group)

    def view(self, layer: int, which: int, m: int) -> torch.Tensor:
        """Local full-width fp16 buffer ``which`` (0 qkvd, 1 h, 2 od, 3 x') of a layer, first m rows."""
        n = (4 * self.stack.hidden, self.stack.inter, 2 * self.stack.hidden, self.stack.hidden)[which]
        o = self.buf[layer][which]
        return self.arena[o:o + self.m_max * n * 2].view(torch.float16).view(self.m_max, n)[:m]

    def _group(self, dests, signal_off: int, done_off: int, wait_off, state_off: int):
        L = self.L
        pg = L.PeerGroup()
        pg.nranks = self.stack.world
        for j, (off, col) in enumerate(dests):
            for p, b in enumerate(self.peers):
                pg.y[j][p] = b + off + col * 2
        for p, b in enumerate(self.peers):
            pg.signal[p] = b + signal_off
        pg.done = self.base + done_off
        pg.wait_count = None if wait_off is None else self.base + wait_off
        pg.wait_state = self.base + state_off
        pg.wait_expected = self.stack.world  # one increment per rank and step
        return pg

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """The sharded decode step on fp16 x [m, hidden] (m <= m_max, replicated); returns the local
        full-width output buffer after every rank's slice of it has arrived."""
        from .quant import _DTYPE_CODE, _stream

        L, st = self.L, self.stack
        m = x.shape[0]
        if m > self.m_max:
            raise ValueError("the peer exchange was laid out for %d rows (got %d)" % (self.m_max, m))
        hd, it, w, r = st.hidden, st.inter, st.world, st.rank
        code, stream = _DTYPE_CODE[x.dtype], _stream(x.device)
        if st.overlap:
            return self._forward_overlapped(x, code, stream)
        cur = x
        for i, layer in enumerate(st.layers):
            q_off, h_off, od_off, x_off = self.buf[i]
            qkvd, h, od, xn = (self.view(i, k, m) for k in range(4))
            hs, qs = it // w, 4 * hd // w
            jobs = [layer.mlp.gateup_job(cur, h[:, r * hs:(r + 1) * hs]), layer.qkvd.gemv_job(cur, qkvd[:, r * qs:(r + 1) * qs])]
            pg = self._group([(h_off, r * hs), (q_off, r * qs)], self.cnt[i][0], self.done[i][0],
                             None if i == 0 else self.cnt[i - 1][1], self.state[i][0])
            L.call("sbq_gemv_w8_group_peer", (L.GemvJob * 2)(*jobs), 2, code, m, ctypes.byref(pg), stream)
            s = hd // w
            jobs = [layer.mlp.down_proj.gemv_job(h, od[:, r * s:(r + 1) * s]),
                    layer.o.gemv_job(qkvd[:, 2 * hd:3 * hd], xn[:, r * s:(r + 1) * s]),
                    layer.dout.gemv_job(qkvd[:, 3 * hd:], od[:, hd + r * s:hd + (r + 1) * s])]
            pg = self._group([(od_off, r * s), (x_off, r * s), (od_off, hd + r * s)], self.cnt[i][1],
                             self.done[i][1], self.cnt[i][0], self.state[i][1])
            L.call("sbq_gemv_w8_group_peer", (L.GemvJob * 3)(*jobs), 3, code, m, ctypes.byref(pg), stream)
            st._side = (od, False)  # stored in place at full width
            cur = xn
        L.call("sbq_peer_wait", ctypes.c_void_p(self.base + self.cnt[-1][1]),
               ctypes.c_void_p(self.base + self.final_state), w, 0, stream)
        return cur

    def _forward_overlapped(self, x: torch.Tensor, code: int, stream) -> torch.Tensor:
        """forward with the side outputs of layer i - 1 as ready jobs of layer i's first launch
        (their inputs are complete on every rank once the o launch in between has seen its signal),
        [o] alone in the second launch, and one last launch for the last layer's side outputs."""
        L, st = self.L, self.stack
        if len(st.layers) == 0:
            return x
        m = x.shape[0]
        hd, it, w, r = st.hidden, st.inter, st.world, st.rank
        hs, qs, s = it // w, 4 * hd // w, hd // w
        cur = x
        for i, layer in enumerate(st.layers):
            q_off, h_off, od_off, x_off = self.buf[i]
            qkvd, h, od, xn = (self.view(i, k, m) for k in range(4))
            jobs, dests = [], []
            if i > 0:
                pq, ph, pod = (self.view(i - 1, k, m) for k in range(3))
                prev, pod_off = st.layers[i - 1], self.buf[i - 1][2]
                jobs += [prev.mlp.down_proj.gemv_job(ph, pod[:, r * s:(r + 1) * s]),
                         prev.dout.gemv_job(pq[:, 3 * hd:], pod[:, hd + r * s:hd + (r + 1) * s])]
                dests += [(pod_off, r * s), (pod_off, hd + r * s)]
            n_ready = len(jobs)
            jobs += [layer.mlp.gateup_job(cur, h[:, r * hs:(r + 1) * hs]),
                     layer.qkvd.gemv_job(cur, qkvd[:, r * qs:(r + 1) * qs])]
            dests += [(h_off, r * hs), (q_off, r * qs)]
            pg = self._group(dests, self.cnt[i][0], self.done[i][0], None if i == 0 else self.cnt[i - 1][1],
                             self.state[i][0])
            L.call("sbq_gemv_w8_group_peer_ready", (L.GemvJob * len(jobs))(*jobs), len(jobs), n_ready, code, m,
                   ctypes.byref(pg), stream)
            pg = self._group([(x_off, r * s)], self.cnt[i][1], self.done[i][1], self.cnt[i][0], self.state[i][1])
            L.call("sbq_gemv_w8_group_peer", (L.GemvJob * 1)(layer.o.gemv_job(qkvd[:, 2 * hd:3 * hd], xn[:, r * s:(r + 1) * s])),
                   1, code, m, ctypes.byref(pg), stream)
            cur = xn
        last, (q_off, h_off, od_off, _) = st.layers[-1], self.buf[-1]
        qkvd, h, od = (self.view(len(st.layers) - 1, k, m) for k in range(3))
        jobs = [last.mlp.down_proj.gemv_job(h, od[:, r * s:(r + 1) * s]),
                last.dout.gemv_job(qkvd[:, 3 * hd:], od[:, hd + r * s:hd + (r + 1) * s])]
        pg = self._group([(od_off, r * s), (od_off, hd + r * s)], self.cnt_last, self.done_last, self.cnt[-1][1],
                         self.state_last)
        L.call("sbq_gemv_w8_group_peer_ready", (L.GemvJob * 2)(*jobs), 2, 2, code, m, ctypes.byref(pg), stream)
        st._side = (od, False)  # stored in place at full width
        L.call("sbq_peer_wait", ctypes.c_void_p(self.base + self.cnt_last),
               ctypes.c_void_p(self.base + self.final_state), w, 0, stream)
        return cur

    def close(self) -> None:
        """Unmap the other ranks' arenas and free this one (every rank, after its last step)."""
        import torch.distributed as dist

        if self.base is None:
            return
        dist.barrier(group=self.stack.group)
        for p, b in enumerate(self.peers):
            if b != self.base:
                self.L.call("sbq_peer_close", ctypes.c_void_p(b))
        self.arena = None
        self.L.call("sbq_peer_free", ctypes.c_void_p(self.base))
        self.base = None


def side_layout(gathered: torch.Tensor | None, world: int, hidden: int) -> torch.Tensor | None:
    """[m, world * 2 * hidden / world] all-gathered [down slice | delta_out slice] blocks of every rank
    -> [m, 2 * hidden] = [down(h) | delta_out(delta_in)] in channel order."""
    if gathered is None or world == 1:
        return gathered
    m = gathered.shape[0]
    return gathered.reshape(m, world, 2, hidden // world).transpose(1, 2).reshape(m, 2 * hidden)


class ProjectionStack(nn.Module):
    """The stack; ``forward(x)`` maps fp16 [m, hidden] to fp16 [m, hidden] on the device."""

    def __init__(self, layers: int = W.LAYERS, hidden: int = W.HIDDEN, inter: int = W.INTER, seed: int = 4,
                 device=None, group=None, exchange: str = "peer", overlap: bool = True):
        super().__init__()
        import torch.distributed as dist

        if exchange not in ("peer", "nccl"):
            raise ValueError("exchange must be 'peer' or 'nccl'")
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
        self.exchange = exchange if self.world > 1 else "none"
        # decode sizes, one GPU or the peer exchange: the side-output projections run as ready jobs
        # of the next layer's first launch
        self.overlap = overlap and self.exchange != "nccl"
        self.peer = PeerExchange(self) if self.exchange == "peer" else None
        self._side = (None, False)  # the last forward's last-layer side outputs, reordered on access?

    @property
    def side(self) -> torch.Tensor | None:
        """The last forward's last-layer side outputs [down(h) | delta_out(delta_in)], full width."""
        t, gathered = self._side
        return side_layout(t, self.world, self.hidden) if gathered else t

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
        (both read x) and [down, o, delta_out] (after their inputs are gathered); o's output is the
        next layer's input.  With ``overlap`` (one GPU, or the peer exchange) the side outputs move to
        the next layer's first launch, as ready jobs whose inputs are two launches old: layer i runs
        [down(h), delta_out of layer i - 1 | gate/up, q|k|v|delta_in] and [o], and one last launch
        computes the last layer's side outputs.  The ready jobs stream while the o launch before them
        ends, so that launch boundary overlaps work (measured at full size: 1.69-1.71 -> 1.65 ms per
        step at batch 1, 2.06 -> 1.94 ms at batch 8 on one GPU; 1.41 -> 1.26 ms at batch 1 on two).
        Above 16 rows (one GEMM per projection) one GPU runs the q|k|v|delta_in -> o chain and the
        other projections on two streams (``_forward_side_stream``).
        """
        if x.shape[0] <= 16:
            if self.peer is not None:
                return self.peer.forward(x)
            return self._forward_grouped(x)
        hd, w = self.hidden, self.world
        m = x.shape[0]
        if self.overlap and w == 1:
            return self._forward_side_stream(x)
        for layer in self.layers:
            qkvd = self._gather(layer.qkvd.forward_into(x, x.new_empty(m, 4 * hd // w)))
            h = self._gather(layer.mlp.gateup_into(x, x.new_empty(m, self.inter // w)))
            od = x.new_empty(m, 2 * hd // w)
            layer.mlp.down_proj.forward_into(h, od[:, :hd // w])
            layer.dout.forward_into(qkvd[:, 3 * hd:], od[:, hd // w:])
            self._side = (self._gather(od), True)
            x = self._gather(layer.o.forward_into(qkvd[:, 2 * hd:3 * hd], x.new_empty(m, hd // w)))
        return x

    def _forward_side_stream(self, x: torch.Tensor) -> torch.Tensor:
        """One GPU above 16 rows (one GEMM launch per projection): the layer chain q|k|v|delta_in ->
        o runs on the caller's stream; gate/up and the side outputs down(h) and delta_out(delta_in),
        which nothing on the chain reads, run on a second stream that waits only for their inputs
        (the layer input, then q|k|v|delta_in), so the two streams fill each other's launch
        boundaries and tails.  The caller's stream joins the second one at the end (also inside a
        CUDA-graph capture: the two streams become parallel branches)."""
        hd, m = self.hidden, x.shape[0]
        main = torch.cuda.current_stream(x.device)
        if getattr(self, "_side_stream", None) is None:
            self._side_stream = torch.cuda.Stream(x.device)
        side = self._side_stream
        keep = []  # tensors read on the second stream stay allocated until the streams join
        od = None
        for layer in self.layers:
            h, qkvd, od = x.new_empty(m, self.inter), x.new_empty(m, 4 * hd), x.new_empty(m, 2 * hd)
            keep += [x, h, qkvd, od]
            side.wait_stream(main)  # the layer input
            with torch.cuda.stream(side):
                layer.mlp.gateup_into(x, h)
            layer.qkvd.forward_into(x, qkvd)
            side.wait_stream(main)  # q|k|v|delta_in
            with torch.cuda.stream(side):
                layer.mlp.down_proj.forward_into(h, od[:, :hd])
                layer.dout.forward_into(qkvd[:, 3 * hd:], od[:, hd:])
            x = layer.o.forward_into(qkvd[:, 2 * hd:3 * hd], x.new_empty(m, hd))
        main.wait_stream(side)
        self._side = (od, False)
        return x

    def forward_modules(self, x: torch.Tensor) -> torch.Tensor:
        """The same data flow through the drop-in's public module calls only (Int8Linear.__call__,
        FusedGatedMLP.__call__ = down(silu(gate(x)) * up(x))), as the reference's model would make
        them: x may be a host tensor (each call then copies its input in and its output back, the
        path a reference model loop on the CPU gets) or a device tensor (stream-ordered, no sync).
        One GPU only."""
        if self.world != 1:
            raise RuntimeError("forward_modules runs an unsharded stack")
        hd = self.hidden
        for layer in self.layers:
            qkvd = layer.qkvd(x)
            side = layer.mlp(x)
            dout = layer.dout(qkvd[:, 3 * hd:])
            x = layer.o(qkvd[:, 2 * hd:3 * hd])
        self._side = (torch.cat([side, dout], 1), False)
        return x

    def _forward_overlapped(self, x: torch.Tensor) -> torch.Tensor:
        from .quant import gemv_group

        hd, m = self.hidden, x.shape[0]
        if len(self.layers) == 0:
            return x
        keep = []  # every buffer stays allocated until the step is enqueued: no launch reuses
        prev = None  # memory that the launch before it may still be reading
        for layer in self.layers:
            qkvd = x.new_empty(m, 4 * hd)
            h = x.new_empty(m, self.inter)
            od = x.new_empty(m, 2 * hd)
            xn = x.new_empty(m, hd)
            keep += [qkvd, h, od, xn]
            ready = [] if prev is None else [prev[0].mlp.down_proj.gemv_job(prev[2], prev[3][:, :hd]),
                                             prev[0].dout.gemv_job(prev[1][:, 3 * hd:], prev[3][:, hd:])]
            gemv_group(ready + [layer.mlp.gateup_job(x, h), layer.qkvd.gemv_job(x, qkvd)], x.dtype, m, x.device,
                       n_ready=len(ready))
            gemv_group([layer.o.gemv_job(qkvd[:, 2 * hd:3 * hd], xn)], x.dtype, m, x.device)
            prev = (layer, qkvd, h, od)
            x = xn
        last, qkvd, h, od = prev
        gemv_group([last.mlp.down_proj.gemv_job(h, od[:, :hd]), last.dout.gemv_job(qkvd[:, 3 * hd:], od[:, hd:])],
                   x.dtype, m, x.device, n_ready=2)
        self._side = (od, False)
        return x

    def _forward_grouped(self, x: torch.Tensor) -> torch.Tensor:
        from .quant import gemv_group

        hd, w = self.hidden, self.world
        m = x.shape[0]
        if self.overlap:
            return self._forward_overlapped(x)
        for layer in self.layers:
            qkvd = x.new_empty(m, 4 * hd // w)
            h = x.new_empty(m, self.inter // w)
            gemv_group([layer.mlp.gateup_job(x, h), layer.qkvd.gemv_job(x, qkvd)], x.dtype, m, x.device)
            qkvd, h = self._gather(qkvd), self._gather(h)
            od = x.new_empty(m, 2 * hd // w)
            xn = x.new_empty(m, hd // w)
            gemv_group([layer.mlp.down_proj.gemv_job(h, od[:, :hd // w]), layer.o.gemv_job(qkvd[:, 2 * hd:3 * hd], xn),
                        layer.dout.gemv_job(qkvd[:, 3 * hd:], od[:, hd // w:])], x.dtype, m, x.device)
            self._side = (self._gather(od), True)
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
            return len(self.layers) * 2 + (1 if self.peer is not None else 0) + (1 if self.overlap else 0)
        return len(self.layers) * 5


class DecodeProgram:
    """A batch-1 decode step of the stack as one launch of the decode program kernel.

    Two stages per layer: [gate/up, q|k|v|delta_in] read the layer input, [down, o, delta_out] read
    their outputs; a grid-wide barrier inside the kernel separates them and the weight stream never
    pauses.  On one GPU every layer gets its own activation buffers (written once per step); a
    sharded stack uses its peer arena (outputs stored to every rank, barriers spanning the ranks).
    ``run()`` reads the fixed input buffer ``x`` and returns the fixed output buffer (the last
    layer's o output, full width).
    """

    def __init__(self, stack: ProjectionStack, x: torch.Tensor):
        from . import _lib as L
        from .quant import _DTYPE_CODE

        if stack.world != 1 and stack.peer is None:
            raise ValueError("a sharded decode program needs the peer exchange")
        if x.shape != (1, stack.hidden) or x.dtype != torch.float16 or not x.is_contiguous():
            raise ValueError("the decode program takes a contiguous fp16 [1, hidden] input")
        hd, dev, w, r = stack.hidden, x.device, stack.world, stack.rank
        self.stack, self.x = stack, x
        self.buffers = []
        jobs, stage, dests = [], [], []
        px = stack.peer
        cur = x
        for i, layer in enumerate(stack.layers):
            if px is None:
                qkvd = torch.empty(1, 4 * hd, dtype=torch.float16, device=dev)
                h = torch.empty(1, stack.inter, dtype=torch.float16, device=dev)
                od = torch.empty(1, 2 * hd, dtype=torch.float16, device=dev)
                nxt = torch.empty(1, hd, dtype=torch.float16, device=dev)
                self.buffers += [qkvd, h, od, nxt]
                sl = lambda t, a, b: t[:, a:b]  # noqa: E731
                hs, qs, s = stack.inter, 4 * hd, hd
            else:
                qkvd, h, od, nxt = (px.view(i, k, 1) for k in range(4))
                sl = lambda t, a, b: t[:, a:b]  # noqa: E731
                hs, qs, s = stack.inter // w, 4 * hd // w, hd // w
            q_off, h_off, od_off, x_off = px.buf[i] if px is not None else (0, 0, 0, 0)
            jobs += [layer.mlp.gateup_job(cur, sl(h, r * hs, (r + 1) * hs)),
                     layer.qkvd.gemv_job(cur, sl(qkvd, r * qs, (r + 1) * qs))]
            dests += [(h_off, r * hs), (q_off, r * qs)]
            stage += [2 * i, 2 * i]
            jobs += [layer.mlp.down_proj.gemv_job(h, sl(od, r * s, (r + 1) * s)),
                     layer.o.gemv_job(qkvd[:, 2 * hd:3 * hd], sl(nxt, r * s, (r + 1) * s)),
                     layer.dout.gemv_job(qkvd[:, 3 * hd:], sl(od, hd + r * s, hd + (r + 1) * s))]
            dests += [(od_off, r * s), (x_off, r * s), (od_off, hd + r * s)]
            stage += [2 * i + 1] * 3
            cur = nxt
        self.y = cur
        self.nstages = 2 * len(stack.layers)
        lib = L.load()
        nbytes = int(lib.sbq_gemv_program_bytes(self.nstages))
        self.program = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        arr = (L.GemvJob * len(jobs))(*jobs)
        st = (ctypes.c_int * len(stage))(*stage)
        self._code = _DTYPE_CODE[torch.float16]
        if px is None:
            self.sync = torch.zeros(int(lib.sbq_gemv_program_sync_bytes(self.nstages)), dtype=torch.uint8, device=dev)
            self._sync_ptr = self.sync.data_ptr()
            L.call("sbq_gemv_program_build", arr, st, len(jobs), self._code, 1,
                   ctypes.c_void_p(self.program.data_ptr()), nbytes)
        else:
            yd = (ctypes.c_void_p * (len(jobs) * w))(*[b + off + col * 2 for off, col in dests for b in px.peers])
            ps = (ctypes.c_void_p * w)(*[b + px.prog_sync for b in px.peers])
            self._sync_ptr = px.base + px.prog_sync
            L.call("sbq_gemv_program_build_peer", arr, st, len(jobs), self._code, 1, yd, w, ps,
                   ctypes.c_void_p(self.program.data_ptr()), nbytes)

    def run(self) -> torch.Tensor:
        from . import _lib as L
        from .quant import _stream

        L.call("sbq_gemv_program_run", ctypes.c_void_p(self.program.data_ptr()), self.nstages, self._code,
               ctypes.c_void_p(self._sync_ptr), _stream(self.x.device))
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
        # grouped launches by default; use_program=True runs a batch-1 step as one decode-program
        # launch (bit-identical)
        self.program = stack.decode_program(self.x) if (m == 1 and use_program) else None
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
