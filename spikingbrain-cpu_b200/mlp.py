"""Fused SwiGLU MLP over int8 projections (GatedMLP.forward, spikingbrain_cpu/model.py:239-240).

The reference runs ``down(silu(gate(x)) * up(x))`` as three Int8Linear calls plus two
elementwise ops.  For decode-sized inputs ``FusedGatedMLP`` streams the gate and up weights in one
kernel (sbq_mlp_gateup_w8), applies SiLU(gate) * up in its epilogue, writes the hidden activation
once (fp16 by default) and runs the down projection on it.  ``fuse_gated_mlp`` swaps the module
in place inside a loaded model.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib as L
from .quant import _DTYPE_CODE, Int8Linear, _prepare_x, _ptr, _stream, _workspace


class FusedGatedMLP(nn.Module):
    def __init__(self, gate: Int8Linear, up: Int8Linear, down: Int8Linear, h_dtype: torch.dtype = torch.float16,
                 shards: int = 1):
        """``shards`` > 1: gate/up hold one output-channel shard each and down consumes the gathered
        activation of all ``shards`` of them (the sharded stack); ``forward`` is then unavailable."""
        super().__init__()
        if not all(isinstance(mod, Int8Linear) for mod in (gate, up, down)):
            raise ValueError("FusedGatedMLP needs int8 gate, up and down projections")
        if gate.bias is not None or up.bias is not None:
            raise ValueError("the fused gate/up epilogue has no bias term")
        if gate.out_features != up.out_features or gate.in_features != up.in_features:
            raise ValueError("gate and up projections must have the same shape")
        if down.in_features != gate.out_features * shards:
            raise ValueError("down projection input must match the gate/up output")
        self.shards = shards
        if h_dtype not in (torch.float16, torch.float32):
            raise ValueError("hidden activation dtype must be float16 or float32")
        self.gate_proj, self.up_proj, self.down_proj = gate, up, down
        self.h_dtype = h_dtype

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.shards != 1:
            raise RuntimeError("a sharded FusedGatedMLP needs the gather between gate/up and down; use the stack")
        shape = x.shape
        dev = self.gate_proj.scale.device
        x2, k16, on_host = _prepare_x(x, self.gate_proj.in_features, dev)
        m, n = x2.shape[0], self.gate_proj.out_features
        h = self.gateup_into(x2, torch.empty(m, n, dtype=self.h_dtype, device=dev))
        y = self.down_proj(h).reshape(*shape[:-1], self.down_proj.out_features)
        return y.to("cpu") if on_host else y

    def gateup_job(self, x2: torch.Tensor, h: torch.Tensor) -> L.GemvJob:
        """silu(gate(x2)) * up(x2) into ``h`` as one job of a grouped decode launch."""
        g, u = self.gate_proj, self.up_proj
        return L.GemvJob(x2.data_ptr(), x2.stride(0), g.packed.data_ptr(), g.scale.data_ptr(), u.packed.data_ptr(),
                         u.scale.data_ptr(), None, g.out_features, x2.shape[1], h.data_ptr(),
                         L.F32 if h.dtype == torch.float32 else L.F16, h.stride(0))

    def gateup_into(self, x2: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
        """Low-level device call: silu(gate(x2)) * up(x2) into ``h`` [m, n] (fp16/fp32, unit column stride).

        x2 is [m, k'] with 16-byte aligned rows (k' = in_features rounded up to 16).  The library
        picks the kernel: the fused gate/up GEMV up to 16 rows; above, the gate GEMM into ``h`` and the
        up GEMM whose epilogue replaces it by silu(gate) * up (fp32 x split once into bf16 high / low
        parts in a workspace that both GEMMs read).
        """
        m, n = x2.shape[0], self.gate_proj.out_features
        if m > 0:
            ws, ws_bytes = _workspace(m, x2.shape[1], x2.dtype, h.device)
            L.call("sbq_mlp_gateup_w8_ws", _ptr(x2), _DTYPE_CODE[x2.dtype], x2.stride(0),
                   _ptr(self.gate_proj.packed), _ptr(self.gate_proj.scale), _ptr(self.up_proj.packed),
                   _ptr(self.up_proj.scale), m, n, x2.shape[1], _ptr(h), L.F16 if h.dtype == torch.float16 else L.F32,
                   h.stride(0), _ptr(ws), ws_bytes, _stream(h.device))
        return h


def fuse_gated_mlp(model: nn.Module, h_dtype: torch.dtype = torch.float16) -> int:
    """Replace every submodule holding int8 ``gate_proj``/``up_proj``/``down_proj`` by FusedGatedMLP.

    Returns how many were replaced.
    """
    count = 0
    for name, mod in list(model.named_modules()):
        if isinstance(mod, FusedGatedMLP):
            continue
        parts = [getattr(mod, a, None) for a in ("gate_proj", "up_proj", "down_proj")]
        if all(isinstance(p, Int8Linear) for p in parts) and parts[0].bias is None and parts[1].bias is None:
            parent_name, _, child = name.rpartition(".")
            parent = model.get_submodule(parent_name) if parent_name else None
            fused = FusedGatedMLP(*parts, h_dtype=h_dtype)
            if parent is None:
                raise ValueError("cannot replace the root module in place")
            setattr(parent, child, fused)
            count += 1
    return count


class FusedLoRAPair(nn.Module):
    """The hybrid block's rank-128 pair (model.py:287-288): ``nn.Sequential(Linear(hidden, 128),
    Linear(128, heads * head_dim))`` with both stages in the int8 format, as one module.

    Up to 16 rows of x run as one launch (sbq_lora_pair_w8: the rank-r intermediate stays on the SMs
    in fp32); more rows run the two projections one after the other (the intermediate in fp32, as
    the reference's Sequential passes it).  Returns fp32 like the reference (``out_dtype`` may be set
    to float16).
    """

    MAX_FUSED_ROWS = 16
    MAX_RANK = 128

    def __init__(self, first: Int8Linear, second: Int8Linear):
        super().__init__()
        if not isinstance(first, Int8Linear) or not isinstance(second, Int8Linear):
            raise ValueError("FusedLoRAPair needs two int8 projections")
        if second.in_features != first.out_features:
            raise ValueError("the second projection must read the first one's output")
        if first.bias is not None or second.bias is not None:
            raise ValueError("the fused pair has no bias terms")
        if first.out_features % 16 or first.out_features > self.MAX_RANK:
            raise ValueError("the pair's inner size must be a multiple of 16 up to %d" % self.MAX_RANK)
        self.first, self.second = first, second
        self.in_features, self.out_features = first.in_features, second.out_features
        self.out_dtype = torch.float32

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        dev = self.first.scale.device
        x2, k16, on_host = _prepare_x(x, self.in_features, dev)
        m = x2.shape[0]
        if m > self.MAX_FUSED_ROWS:
            t = self.first.forward_into(x2, torch.empty(m, self.first.out_features, device=dev))
            y = self.second.forward_into(t, torch.empty(m, self.out_features, dtype=self.out_dtype, device=dev))
        else:
            y = torch.empty(m, self.out_features, dtype=self.out_dtype, device=dev)
            if m > 0:
                L.call("sbq_lora_pair_w8", _ptr(x2), _DTYPE_CODE[x2.dtype], x2.stride(0), _ptr(self.first.packed),
                       _ptr(self.first.scale), _ptr(self.second.packed), _ptr(self.second.scale), m,
                       self.first.out_features, self.out_features, x2.shape[1], _ptr(y),
                       L.F32 if y.dtype == torch.float32 else L.F16, y.stride(0), _stream(dev))
        y = y.reshape(*shape[:-1], self.out_features)
        return y.to("cpu") if on_host else y


def fuse_lora_pairs(model: nn.Module) -> int:
    """Replace every ``nn.Sequential`` of two int8 projections whose inner size fits the fused kernel
    (the LoRA pairs) by a FusedLoRAPair; returns how many were replaced."""
    count = 0
    for name, mod in list(model.named_modules()):
        if not (isinstance(mod, nn.Sequential) and len(mod) == 2):
            continue
        a, b = mod[0], mod[1]
        if not (isinstance(a, Int8Linear) and isinstance(b, Int8Linear)) or a.bias is not None or b.bias is not None:
            continue
        if b.in_features != a.out_features or a.out_features % 16 or a.out_features > FusedLoRAPair.MAX_RANK:
            continue
        parent_name, _, child = name.rpartition(".")
        if not name:
            raise ValueError("cannot replace the root module in place")
        parent = model.get_submodule(parent_name) if parent_name else model
        setattr(parent, child, FusedLoRAPair(a, b))
        count += 1
    return count
