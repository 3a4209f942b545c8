"""Shared-input projection groups: several int8 projections that read the same x, run as one launch.

In the reference's hybrid block every projection of ``sse_inputs`` and of ``swa`` reads the same
activation x (spikingbrain_cpu/model.py:317-333 and :363-365: sse_q/k/v, the first stage of the
lora_q/lora_k pairs, sse_a/b/e, swa_q/k/v), and each is its own ``Int8Linear`` call.
``SharedInputGroup`` concatenates their packed weights along the output channels (each member's
rows padded to a 16-row tile, zero scale on the padding) so that one decode GEMV or one prefill GEMM
streams them all with a single read of x and one launch.  ``fuse_shared_inputs`` puts
``GroupMember`` modules in the members' places: the first member called with a given x runs the
whole group, the others return their slice of that result, so the reference's model code runs
unchanged.  A result is handed out once per computation; a member called again (or with another
x) recomputes.  Members' outputs are column views of the group's [m, padded N] result.

Both int8 formats are supported (all members of one group share the format).  int8-dyn members
give bit-identical results to separate calls: the per-tensor activation quantisation depends on x
only, and each output channel's integer dot product does not depend on its neighbours.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from . import _lib as L
from .quant import DynamicInt8Linear, Int8Linear, _DTYPE_CODE, _prepare_x, _ptr, _stream, _workspace


class SharedInputGroup(nn.Module):
    def __init__(self, members: list[nn.Module]):
        super().__init__()
        if not members:
            raise ValueError("a group needs at least one projection")
        kind = type(members[0])
        if kind not in (Int8Linear, DynamicInt8Linear) or any(type(m) is not kind for m in members):
            raise ValueError("group members must all be Int8Linear or all DynamicInt8Linear")
        k = members[0].in_features
        if any(m.in_features != k for m in members):
            raise ValueError("group members must read the same input width")
        if kind is DynamicInt8Linear and len({m.mode for m in members}) != 1:
            raise ValueError("group members must share the activation quantisation mode")
        dev = members[0].scale.device
        self.kind, self.in_features = kind, k
        self.sizes = [m.out_features for m in members]
        self.offsets, off = [], 0
        for n in self.sizes:
            self.offsets.append(off)
            off += (n + 15) // 16 * 16
        self.n_pad = off
        kt = (k + 63) // 64
        packed = torch.zeros(L.packed_bytes(self.n_pad, k), dtype=torch.int8, device=dev)
        scale = torch.zeros(self.n_pad, dtype=torch.float32, device=dev)
        has_bias = any(m.bias is not None for m in members)
        bias = torch.zeros(self.n_pad, dtype=torch.float32, device=dev) if has_bias else None
        rowsum = torch.zeros(self.n_pad, dtype=torch.int32, device=dev) if kind is DynamicInt8Linear else None
        for m, o, n in zip(members, self.offsets, self.sizes):
            b0 = (o // 16) * kt * 1024  # the member's tile-rows, contiguous in the packed layout
            packed[b0:b0 + m.packed.numel()].copy_(m.packed)
            scale[o:o + n].copy_(m.scale)
            if m.bias is not None:
                bias[o:o + n].copy_(m.bias)
            if rowsum is not None:
                rowsum[o:o + n].copy_(m.rowsum)
        self.register_buffer("packed", packed, persistent=False)
        self.register_buffer("scale", scale, persistent=False)
        self.register_buffer("bias", bias, persistent=False)
        self.register_buffer("rowsum", rowsum, persistent=False)
        self.mode = getattr(members[0], "mode", None)
        self.out_dtype = torch.float32
        self._result = None
        self._key = None
        self._handed = set()

    def forward_all(self, x: torch.Tensor) -> list[torch.Tensor]:
        """Every member's output for x [..., k] (one launch sequence); a list of column views."""
        shape = x.shape
        dev = self.scale.device
        x2, k16, on_host = _prepare_x(x, self.in_features, dev)
        m = x2.shape[0]
        out = torch.empty(m, self.n_pad, dtype=self.out_dtype, device=dev)
        if m > 0:
            st = _stream(dev)
            if self.kind is Int8Linear:
                ws, ws_bytes = _workspace(m, x2.shape[1], x2.dtype, dev)
                L.call("sbq_linear_w8_ws", _ptr(x2), _DTYPE_CODE[x2.dtype], x2.stride(0), _ptr(self.packed),
                       _ptr(self.scale), _ptr(self.bias), m, self.n_pad, x2.shape[1], _ptr(out),
                       L.F32 if out.dtype == torch.float32 else L.F16, out.stride(0), _ptr(ws), ws_bytes, st)
            else:
                code = L.ACT_PER_TENSOR if self.mode == "per_tensor" else L.ACT_PER_TOKEN
                ws_bytes = int(L.load().sbq_dyn_workspace_bytes(m, k16, code))
                ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
                L.call("sbq_linear_dyn", _ptr(x2), _DTYPE_CODE[x2.dtype], x2.stride(0), code, _ptr(self.packed),
                       _ptr(self.rowsum), _ptr(self.scale), _ptr(self.bias), m, self.n_pad, k16, _ptr(out),
                       self.n_pad, _ptr(ws), ws_bytes, st)
        if on_host:
            out = out.to("cpu")
        out = out.reshape(*shape[:-1], self.n_pad)
        return [out[..., o:o + n] for o, n in zip(self.offsets, self.sizes)]

    def member_output(self, index: int, x: torch.Tensor) -> torch.Tensor:
        key = (id(x), x.data_ptr(), x._version, tuple(x.shape), x.dtype, x.device)
        if self._result is None or self._key != key or index in self._handed:
            self._result = self.forward_all(x)
            self._key = key
            self._handed = set()
        self._handed.add(index)
        return self._result[index]


class GroupMember(nn.Module):
    """Stands in a group member's place; calling it returns that member's output (see module doc)."""

    def __init__(self, group: SharedInputGroup, index: int):
        super().__init__()
        self.index = index
        self.out_features = group.sizes[index]
        self.in_features = group.in_features
        object.__setattr__(self, "group", group)  # shared, not a child module of every member

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.group.member_output(self.index, x)


def fuse_shared_inputs(parent: nn.Module, names: list[str]) -> SharedInputGroup:
    """Replace the int8 submodules ``names`` of ``parent`` (dotted paths, e.g. ``"lora_q_proj.0"``)
    by members of one SharedInputGroup; returns the group (also kept as ``parent.shared_input_group``
    or ``shared_input_group_<i>``)."""
    mods = [parent.get_submodule(n) for n in names]
    group = SharedInputGroup(mods)
    for i, n in enumerate(names):
        owner_name, _, leaf = n.rpartition(".")
        owner = parent.get_submodule(owner_name) if owner_name else parent
        setattr(owner, leaf, GroupMember(group, i))
    attr, i = "shared_input_group", 0
    while hasattr(parent, attr):
        i += 1
        attr = "shared_input_group_%d" % i
    setattr(parent, attr, group)
    return group


# The projections of one hybrid block (spikingbrain_cpu/model.py HybridSSEAttention) that read x.
HYBRID_SHARED_INPUTS = ["sse_q_proj", "sse_k_proj", "sse_v_proj", "lora_q_proj.0", "lora_k_proj.0", "sse_a_proj",
                        "sse_b_proj", "sse_e_proj", "swa_q_proj", "swa_k_proj", "swa_v_proj"]
# The same for a softmax-attention block (model.py SoftmaxAttention).
ATTENTION_SHARED_INPUTS = ["q_proj", "k_proj", "v_proj"]
