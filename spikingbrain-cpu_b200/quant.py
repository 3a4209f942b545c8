"""Drop-in replacement for spikingbrain_cpu/quant.py on B200 (sm_100a).

Same public surface as the reference module: ``FORMATS``, ``quantize_per_channel``,
``Int8Linear(weight, bias, block=128)``, ``DynamicInt8Linear(weight, bias)``, the float formats
and ``make_linear(fmt, weight, bias=None)`` (quant.py:22-111).  Modules take the weight the
loader hands them (a CPU bf16/fp32 tensor, loader.py:49), quantise and pack it on the current
CUDA device once, and own the device buffers.  ``forward`` returns fp32 like the reference.

The ``int8`` and ``int8-dyn`` formats run only through libsbq.so (hand-written sm_100a kernels);
there is no CPU or PyTorch fallback for them.  A CPU input tensor is copied to the device, run
there and the result copied back, so the modules also work inside the reference's CPU model
loop; device inputs stay on the device with no host synchronisation.
"""

from __future__ import annotations

import ctypes

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib as L

FORMATS = ("float32", "bfloat16", "float16", "int8", "int8-dyn")

_DTYPE_CODE = {torch.float32: L.F32, torch.float16: L.F16, torch.bfloat16: L.BF16}
_ELEM = {torch.float32: 4, torch.float16: 2, torch.bfloat16: 2}


def _device(device=None) -> torch.device:
    if device is not None:
        device = torch.device(device)
        if device.type != "cuda":
            raise ValueError("int8 formats run on a CUDA device, got " + str(device))
        return device
    if not torch.cuda.is_available():
        raise RuntimeError("the int8 formats need a CUDA device (B200, sm_100a); none is available")
    return torch.device("cuda", torch.cuda.current_device())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _ptr(t: torch.Tensor | None):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def pack_weight(weight: torch.Tensor, device=None, rowsum: bool = False):
    """Quantise an [n, k] float weight per output channel on the device (quant.py:25-29) and pack it.

    Returns ``(packed, scale, rowsum)``: the packed int8 tiles (flat int8 tensor), the fp32
    per-row scales and, if asked for, the int32 row sums used by the int8-dyn epilogue.
    """
    dev = _device(device)
    if weight.dim() != 2:
        raise ValueError("weight must be 2-D [out_features, in_features], got shape %s" % (tuple(weight.shape),))
    w = weight.detach()
    if w.dtype not in _DTYPE_CODE:
        w = w.float()
    w = w.to(dev)
    if w.stride(1) != 1 or w.stride(0) < w.shape[1]:
        w = w.contiguous()
    n, k = w.shape
    packed = torch.empty(L.packed_bytes(n, k), dtype=torch.int8, device=dev)
    scale = torch.empty(n, dtype=torch.float32, device=dev)
    rs = torch.empty(n, dtype=torch.int32, device=dev) if rowsum else None
    L.call("sbq_quantize_pack", _ptr(w), _DTYPE_CODE[w.dtype], n, k, w.stride(0), _ptr(packed), _ptr(scale),
           _ptr(rs), _stream(dev))
    return packed, scale, rs


def pack_int8(q: torch.Tensor, device=None, rowsum: bool = False):
    """Pack an already-quantised int8 [n, k] weight (e.g. a ``qweight`` from a state dict)."""
    dev = _device(device)
    if q.dim() != 2 or q.dtype != torch.int8:
        raise ValueError("qweight must be a 2-D int8 tensor")
    q = q.to(dev).contiguous()
    n, k = q.shape
    packed = torch.empty(L.packed_bytes(n, k), dtype=torch.int8, device=dev)
    rs = torch.empty(n, dtype=torch.int32, device=dev) if rowsum else None
    L.call("sbq_pack_int8", _ptr(q), n, k, k, _ptr(packed), _ptr(rs), _stream(dev))
    return packed, rs


def unpack_int8(packed: torch.Tensor, n: int, k: int) -> torch.Tensor:
    """Packed tiles -> row-major int8 [n, k] on the same device."""
    q = torch.empty(n, k, dtype=torch.int8, device=packed.device)
    L.call("sbq_unpack_int8", _ptr(packed), n, k, _ptr(q), k, _stream(packed.device))
    return q


def quantize_per_channel(weight: torch.Tensor, device=None) -> tuple[torch.Tensor, torch.Tensor]:
    """quant.py:25-29 computed on the device: ``(q int8 [n, k], scale fp32 [n])``, bit-identical."""
    packed, scale, _ = pack_weight(weight, device)
    return unpack_int8(packed, *weight.shape), scale


def _workspace(m: int, k: int, x_dtype: torch.dtype, device: torch.device):
    """(workspace tensor or None, bytes) for the int8 format's fp32 prefill path (sbq_linear_w8_ws):
    the bf16 high / low parts of x, taken from torch's caching allocator (no device sync)."""
    nbytes = int(L.load().sbq_linear_w8_workspace_bytes(m, k, _DTYPE_CODE[x_dtype]))
    if nbytes == 0:
        return None, 0
    return torch.empty(nbytes, dtype=torch.uint8, device=device), nbytes


def _prepare_x(x: torch.Tensor, k: int, device: torch.device):
    """Flatten x to [m, k'] on the device with 16-byte aligned rows; k' is k rounded up to 16."""
    if x.shape[-1] != k:
        raise ValueError("input feature size %d does not match the weight's %d" % (x.shape[-1], k))
    on_host = x.device.type != "cuda"
    xd = x.to(device, non_blocking=True) if on_host or x.device != device else x
    if xd.dtype not in _DTYPE_CODE:
        xd = xd.float()
    x2 = xd.reshape(-1, k)
    k16 = (k + 15) // 16 * 16
    if k16 != k:
        x2 = F.pad(x2, (0, k16 - k))
    elif (x2.stride(-1) != 1 or (x2.stride(0) * _ELEM[x2.dtype]) % 16 or x2.data_ptr() % 16) and x2.shape[0] > 0:
        x2 = x2.contiguous()
    return x2, k16, on_host


class _PackedLinear(nn.Module):
    """Common state handling: device-packed weight, reference-compatible state dict keys."""

    def _init_packed(self, weight: torch.Tensor, bias: torch.Tensor | None, device, rowsum: bool):
        dev = _device(device)
        packed, scale, rs = pack_weight(weight, dev, rowsum=rowsum)
        self.out_features, self.in_features = int(weight.shape[0]), int(weight.shape[1])
        self.register_buffer("packed", packed, persistent=False)
        self.register_buffer("scale", scale)
        if rowsum:
            self.register_buffer("rowsum", rs, persistent=False)
        else:
            self.rowsum = None
        self.bias = None if bias is None else nn.Parameter(bias.detach().float().to(dev), requires_grad=False)

    @classmethod
    def from_packed(cls, packed: torch.Tensor, scale: torch.Tensor, rowsum: torch.Tensor | None, out_features: int,
                    in_features: int, bias: torch.Tensor | None = None, **attrs):
        """A module around weights already quantised and packed on the device (e.g. by
        ``loader.StreamingPacker``); the buffers are adopted, not copied."""
        if packed.numel() != L.packed_bytes(out_features, in_features) or scale.numel() != out_features:
            raise ValueError("packed buffers do not match a [%d, %d] weight" % (out_features, in_features))
        mod = cls.__new__(cls)
        nn.Module.__init__(mod)
        mod.out_features, mod.in_features = int(out_features), int(in_features)
        mod.register_buffer("packed", packed, persistent=False)
        mod.register_buffer("scale", scale)
        if rowsum is not None:
            mod.register_buffer("rowsum", rowsum, persistent=False)
        else:
            mod.rowsum = None
        dev = scale.device
        mod.bias = None if bias is None else nn.Parameter(bias.detach().float().to(dev), requires_grad=False)
        for k_, v in attrs.items():
            setattr(mod, k_, v)
        return mod

    @property
    def qweight(self) -> torch.Tensor:
        """Row-major int8 [out, in] view of the packed weight (the reference's ``qweight`` buffer)."""
        return unpack_int8(self.packed, self.out_features, self.in_features)

    def _save_to_state_dict(self, destination, prefix, keep_vars):
        super()._save_to_state_dict(destination, prefix, keep_vars)
        destination[prefix + "qweight"] = self.qweight

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        key = prefix + "qweight"
        q = state_dict.get(key)
        super()._load_from_state_dict(state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                                      error_msgs)
        if key in unexpected_keys:
            unexpected_keys.remove(key)
        if q is None:
            if strict:
                missing_keys.append(key)
            return
        if tuple(q.shape) != (self.out_features, self.in_features):
            error_msgs.append("size mismatch for %s: %s != %s" % (key, tuple(q.shape),
                                                                  (self.out_features, self.in_features)))
            return
        packed, rs = pack_int8(q, self.packed.device, rowsum=self.rowsum is not None)
        self.packed.copy_(packed)
        if rs is not None:
            self.rowsum.copy_(rs)

    def extra_repr(self) -> str:
        return "in_features=%d, out_features=%d, bias=%s" % (self.in_features, self.out_features, self.bias is not None)


class Int8Linear(_PackedLinear):
    """Format ``int8``: symmetric per-output-channel int8 weight, fp32 scale epilogue (quant.py:32-53).

    ``block`` is accepted for signature compatibility; the device kernels do not dequantise the
    weight into fp32 blocks.  ``out_dtype`` may be set to ``torch.float16`` for the fp16-output
    prefill configuration; the default matches the reference (fp32).
    """

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None, block: int = 128, device=None):
        super().__init__()
        self._init_packed(weight, bias, device, rowsum=False)
        self.block = block
        self.out_dtype = torch.float32

    def forward_into(self, x2: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """Low-level device call: x2 [m, k'] (k' = in_features rounded up to 16, 16-byte aligned rows)
        into ``out`` [m, out_features] (fp32 or fp16, unit column stride, any row stride)."""
        m, n = x2.shape[0], self.out_features
        if out.shape != (m, n) or out.stride(1) != 1 or out.dtype not in (torch.float32, torch.float16):
            raise ValueError("output must be an fp32/fp16 [%d, %d] view with unit column stride" % (m, n))
        if m > 0:
            ws, ws_bytes = _workspace(m, x2.shape[1], x2.dtype, out.device)
            L.call("sbq_linear_w8_ws", _ptr(x2), _DTYPE_CODE[x2.dtype], x2.stride(0), _ptr(self.packed),
                   _ptr(self.scale), _ptr(self.bias), m, n, x2.shape[1], _ptr(out),
                   L.F32 if out.dtype == torch.float32 else L.F16, out.stride(0), _ptr(ws), ws_bytes,
                   _stream(out.device))
        return out

    def gemv_job(self, x2: torch.Tensor, out: torch.Tensor) -> L.GemvJob:
        """This projection as one job of a grouped decode launch (see ``gemv_group``)."""
        return L.GemvJob(x2.data_ptr(), x2.stride(0), self.packed.data_ptr(), self.scale.data_ptr(), None, None,
                         None if self.bias is None else self.bias.data_ptr(), self.out_features, x2.shape[1],
                         out.data_ptr(), L.F32 if out.dtype == torch.float32 else L.F16, out.stride(0))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        dev = self.scale.device
        x2, _, on_host = _prepare_x(x, self.in_features, dev)
        out = torch.empty(x2.shape[0], self.out_features, dtype=self.out_dtype, device=dev)
        self.forward_into(x2, out)
        out = out.reshape(*shape[:-1], self.out_features)
        return out.to("cpu") if on_host else out


def gemv_group(jobs, x_dtype: torch.dtype, m: int, device: torch.device, n_ready: int = 0) -> None:
    """Run several decode projections (``Int8Linear.gemv_job`` / ``FusedGatedMLP.gateup_job``) in one
    launch: up to 8 jobs, all with ``m`` <= 16 rows of x of dtype ``x_dtype``.  The first ``n_ready``
    jobs read inputs written two or more launches back and run without waiting for the previous
    launch (sbq_gemv_w8_group_ready: the previous kernel must be a grouped GEMV launch)."""
    arr = (L.GemvJob * len(jobs))(*jobs)
    if n_ready:
        L.call("sbq_gemv_w8_group_ready", arr, len(jobs), n_ready, _DTYPE_CODE[x_dtype], m, _stream(device))
    else:
        L.call("sbq_gemv_w8_group", arr, len(jobs), _DTYPE_CODE[x_dtype], m, _stream(device))


class DynamicInt8Linear(_PackedLinear):
    """Format ``int8-dyn`` (quant.py:56-66): activations quantised at run time, int8 x int8 -> int32.

    ``mode="per_tensor"`` (default) reproduces the reference bit for bit: fbgemm's per-tensor
    uint8 quantisation with a zero point, int32 accumulation and the fp32 epilogue.
    ``mode="per_token"`` is the symmetric per-row variant (no reference counterpart).
    """

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None, mode: str = "per_tensor", device=None):
        super().__init__()
        if mode not in ("per_tensor", "per_token"):
            raise ValueError("unknown activation quantisation mode " + mode)
        self._init_packed(weight, bias, device, rowsum=True)
        self.mode = mode

    @property
    def _mode_code(self) -> int:
        return L.ACT_PER_TENSOR if self.mode == "per_tensor" else L.ACT_PER_TOKEN

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        dev = self.scale.device
        x2, k16, on_host = _prepare_x(x, self.in_features, dev)
        m, n = x2.shape[0], self.out_features
        out = torch.empty(m, n, dtype=torch.float32, device=dev)
        if m > 0:
            lib = L.load()
            ws_bytes = int(lib.sbq_dyn_workspace_bytes(m, k16, self._mode_code))
            ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
            L.call("sbq_linear_dyn", _ptr(x2), _DTYPE_CODE[x2.dtype], x2.stride(0), self._mode_code,
                   _ptr(self.packed), _ptr(self.rowsum), _ptr(self.scale), _ptr(self.bias), m, n, k16, _ptr(out), n,
                   _ptr(ws), ws_bytes, _stream(dev))
        out = out.reshape(*shape[:-1], n)
        return out.to("cpu") if on_host else out

    def forward_stages(self, x: torch.Tensor):
        """The integer stages separately: ``(y, xq, s, zp, acc)`` (per-token: ``(y, xq, s_tok, None, acc)``).

        Runs the two kernels of ``forward`` through their own entry points and also returns the
        quantised activation, its parameters and the int32 accumulators for bit-exact checks.
        """
        dev = self.scale.device
        x2, k16, _ = _prepare_x(x, self.in_features, dev)
        m, n = x2.shape[0], self.out_features
        st = _stream(dev)
        lib = L.load()
        acc = torch.empty(m, n, dtype=torch.int32, device=dev)
        y = torch.empty(m, n, dtype=torch.float32, device=dev)
        if self.mode == "per_tensor":
            xq = torch.empty(m, k16, dtype=torch.uint8, device=dev)
            s = torch.empty(1, dtype=torch.float32, device=dev)
            zp = torch.empty(1, dtype=torch.int32, device=dev)
            ws_bytes = int(lib.sbq_dyn_workspace_bytes(m, k16, L.ACT_PER_TENSOR))
            ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
            L.call("sbq_quant_act_per_tensor", _ptr(x2), _DTYPE_CODE[x2.dtype], x2.stride(0), m, k16, _ptr(xq),
                   _ptr(s), _ptr(zp), _ptr(ws), ws_bytes, st)
        else:
            xq = torch.empty(m, k16, dtype=torch.int8, device=dev)
            s = torch.empty(m, dtype=torch.float32, device=dev)
            zp = None
            L.call("sbq_quant_act_per_token", _ptr(x2), _DTYPE_CODE[x2.dtype], x2.stride(0), m, k16, _ptr(xq),
                   _ptr(s), st)
        L.call("sbq_gemm_w8a8", _ptr(xq), self._mode_code, _ptr(self.packed), _ptr(self.rowsum), _ptr(s), _ptr(zp),
               _ptr(self.scale), _ptr(self.bias), m, n, k16, _ptr(y), n, _ptr(acc), st)
        return y, xq[:, :self.in_features], s, zp, acc


# ---- float formats (outside the int8 hot path; cuBLAS through torch, fp32 results) ----------

class FP16Linear(nn.Module):
    """Format ``float16`` (quant.py:69-77): fp16 weights, fp32 activations and output."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None, device=None):
        super().__init__()
        dev = _device(device)
        self.register_buffer("weight", weight.detach().to(dev, torch.float16).contiguous())
        self.bias = None if bias is None else nn.Parameter(bias.detach().float().to(dev), requires_grad=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        on_host = x.device.type != "cuda"
        xd = x.to(self.weight.device).float()
        out = torch.matmul(xd, self.weight.t().float())
        if self.bias is not None:
            out = out + self.bias
        return out.to("cpu") if on_host else out


class BF16Linear(nn.Module):
    """Format ``bfloat16`` (quant.py:80-87)."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None, device=None):
        super().__init__()
        dev = _device(device)
        self.register_buffer("weight", weight.detach().to(dev, torch.bfloat16).contiguous())
        self.bias = None if bias is None else nn.Parameter(bias.detach().to(dev, torch.bfloat16), requires_grad=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        on_host = x.device.type != "cuda"
        out = F.linear(x.to(self.weight.device, torch.bfloat16), self.weight, self.bias).float()
        return out.to("cpu") if on_host else out


class FloatLinear(nn.Module):
    """Format ``float32`` (quant.py:90-97)."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None, device=None):
        super().__init__()
        dev = _device(device)
        self.register_buffer("weight", weight.detach().to(dev, torch.float32).contiguous())
        self.bias = None if bias is None else nn.Parameter(bias.detach().float().to(dev), requires_grad=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        on_host = x.device.type != "cuda"
        out = F.linear(x.to(self.weight.device).float(), self.weight, self.bias)
        return out.to("cpu") if on_host else out


def make_linear(fmt: str, weight: torch.Tensor, bias: torch.Tensor | None = None) -> nn.Module:
    """quant.py:100-111: format string -> module; ``ValueError`` for an unknown format."""
    if fmt == "float32":
        return FloatLinear(weight, bias)
    if fmt == "bfloat16":
        return BF16Linear(weight, bias)
    if fmt == "float16":
        return FP16Linear(weight, bias)
    if fmt == "int8":
        return Int8Linear(weight, bias)
    if fmt == "int8-dyn":
        return DynamicInt8Linear(weight, bias)
    raise ValueError("unknown weight format " + fmt)
