"""Streaming quantise-and-pack of checkpoint weights on the GPU (the loader's side of the int8 path).

The reference's loader reads the checkpoint one shard at a time and hands every ``nn.Linear``
weight to ``make_linear(fmt, tensor, None)`` as soon as it is read (spikingbrain_cpu/loader.py:46-51,
:74-88), so a full-precision copy of the model never exists; for ``int8`` / ``int8-dyn`` that call
quantises on the CPU (quant.py:25-29, :57-61).  ``StreamingPacker.make_linear`` takes the same
arguments in the same order and returns the same modules, but each weight is copied into one of two
pinned staging buffers on the host, sent to the GPU on a copy stream and quantised + packed there
(sbq_quantize_pack, bit-identical to quant.py:25-29) on a second stream, while the host already
stages the next weight.  The host tensor may be freed as soon as the call returns.  Weights larger
than a staging buffer go through in row blocks (multiples of 16 rows, one packed tile-row strip
each).  ``finish()`` waits for the last weight; the modules are stream-ordered after it anyway.
"""

from __future__ import annotations

import ctypes

import torch
import torch.nn as nn

from . import _lib as L
from .quant import _DTYPE_CODE, DynamicInt8Linear, Int8Linear, _device, _ptr
from .quant import make_linear as _make_linear_eager


class StreamingPacker:
    def __init__(self, device=None, staging_bytes: int = 256 << 20):
        self.device = _device(device)
        if staging_bytes < 1 << 20:
            raise ValueError("staging buffers of at least 1 MiB")
        self.staging_bytes = int(staging_bytes)
        self.host = [torch.empty(self.staging_bytes, dtype=torch.uint8).pin_memory() for _ in range(2)]
        self.dev = [torch.empty(self.staging_bytes, dtype=torch.uint8, device=self.device) for _ in range(2)]
        self.copy_stream = torch.cuda.Stream(self.device)
        self.pack_stream = torch.cuda.Stream(self.device)
        # per staging slot: host copy may be overwritten (DMA done) / device copy may be overwritten (pack done)
        self.dma_done = [None, None]
        self.pack_done = [None, None]
        self.slot = 0
        self.weights = 0
        self.bytes_in = 0

    def _stage(self, rows: torch.Tensor, packed: torch.Tensor, scale: torch.Tensor, rowsum, row0: int):
        """One block of rows [r, k] of a weight: host -> pinned -> device -> quantise + pack."""
        i = self.slot
        self.slot ^= 1
        nbytes = rows.numel() * rows.element_size()
        if self.dma_done[i] is not None:
            self.dma_done[i].synchronize()  # the pinned buffer's previous contents have left the host
        hv = self.host[i][:nbytes].view(rows.dtype).view(rows.shape)
        hv.copy_(rows)
        dv = self.dev[i][:nbytes].view(rows.dtype).view(rows.shape)
        with torch.cuda.stream(self.copy_stream):
            if self.pack_done[i] is not None:
                self.copy_stream.wait_event(self.pack_done[i])  # the device buffer's previous block is packed
            dv.copy_(hv, non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(self.copy_stream)
            self.dma_done[i] = ev
        self.pack_stream.wait_event(self.dma_done[i])
        n_blk, k = rows.shape
        kt = (k + 63) // 64
        off = (row0 // 16) * kt * 1024
        L.call("sbq_quantize_pack", _ptr(dv), _DTYPE_CODE[rows.dtype], n_blk, k, k, _ptr(packed[off:]),
               _ptr(scale[row0:]), None if rowsum is None else _ptr(rowsum[row0:]),
               ctypes.c_void_p(self.pack_stream.cuda_stream))
        ev = torch.cuda.Event()
        ev.record(self.pack_stream)
        self.pack_done[i] = ev
        self.bytes_in += nbytes

    def pack(self, weight: torch.Tensor, rowsum: bool = False):
        """Quantise + pack one host weight [n, k]; returns (packed, scale, rowsum) device tensors,
        valid on the current stream once it has waited for ``ready_event()`` (make_linear does)."""
        if weight.dim() != 2:
            raise ValueError("weight must be 2-D [out_features, in_features], got shape %s" % (tuple(weight.shape),))
        w = weight.detach()
        if w.dtype not in _DTYPE_CODE:
            w = w.float()
        if w.device.type != "cpu":
            raise ValueError("the streaming packer takes host tensors (got %s)" % w.device)
        w = w.contiguous()
        n, k = w.shape
        dev = self.device
        # the outputs belong to the caller's stream (where the modules will use and free them); the
        # pack stream is ordered after their allocation
        packed = torch.empty(L.packed_bytes(n, k), dtype=torch.int8, device=dev)
        scale = torch.empty(n, dtype=torch.float32, device=dev)
        rs = torch.empty(n, dtype=torch.int32, device=dev) if rowsum else None
        self.pack_stream.wait_stream(torch.cuda.current_stream(dev))
        row_bytes = k * w.element_size()
        blk = max(16, (self.staging_bytes // row_bytes) // 16 * 16)
        if 16 * row_bytes > self.staging_bytes:
            raise ValueError("a 16-row block of this weight (%d bytes) exceeds the staging buffer" % (16 * row_bytes))
        for r0 in range(0, n, blk):
            self._stage(w[r0:r0 + blk], packed, scale, rs, r0)
        self.weights += 1
        return packed, scale, rs

    def ready_event(self) -> torch.cuda.Event:
        ev = torch.cuda.Event()
        ev.record(self.pack_stream)
        return ev

    def make_linear(self, fmt: str, weight: torch.Tensor, bias: torch.Tensor | None = None) -> nn.Module:
        """quant.make_linear's signature and results (quant.py:100-111); int8 formats streamed."""
        if fmt not in ("int8", "int8-dyn"):
            if fmt in ("float32", "bfloat16", "float16"):
                return _make_linear_eager(fmt, weight, bias)
            raise ValueError("unknown weight format " + fmt)
        dyn = fmt == "int8-dyn"
        packed, scale, rs = self.pack(weight, rowsum=dyn)
        torch.cuda.current_stream(self.device).wait_event(self.ready_event())
        n, k = weight.shape
        if dyn:
            return DynamicInt8Linear.from_packed(packed, scale, rs, n, k, bias, mode="per_tensor")
        return Int8Linear.from_packed(packed, scale, None, n, k, bias, block=128, out_dtype=torch.float32)

    def finish(self) -> None:
        """Wait until every weight handed in so far is packed (call it before dropping the packer:
        its staging buffers are in use until then)."""
        self.copy_stream.synchronize()
        self.pack_stream.synchronize()


__all__ = ["StreamingPacker"]
