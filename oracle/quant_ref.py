"""numpy + C restatement of the reference's quantised-linear arithmetic.

TEST INFRASTRUCTURE ONLY (see ``oracle/__init__.py``): this is the checker the
CUDA path is compared against, never part of the product path.

Reference functions restated (paths relative to the reference project):

* ``quantize_per_channel``  spikingbrain_cpu/quant.py:25-29
* ``int8_linear``           Int8Linear.forward, spikingbrain_cpu/quant.py:41-53.
  The reference multiplies fp32 activations by 128-row blocks of the
  dequantised weight with an fp32 sgemm, concatenates the blocks and applies the
  per-row scale after the dot product.  Here the dot product runs in float64 and
  the scale is applied after it, so the oracle is the exact-arithmetic value the
  fp32 reference approximates; parity is a relative-L2 tolerance.
* ``dyn_*``                 DynamicInt8Linear.forward, spikingbrain_cpu/quant.py:63-66
  (torch ``quantized::linear_dynamic`` on the fbgemm/x86 engine), restated
  step by step in ``oracle/dyn_int8.c``.  Bit-exact.
* ``gated_mlp``             GatedMLP.forward, spikingbrain_cpu/model.py:239-240.

Parity is pinned by ``tests/golden`` fixtures produced by running the reference
itself (``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import build as _build

_LIB = None


def lib() -> ctypes.CDLL:
    """Load (building first if needed) the C half of the oracle."""
    global _LIB
    if _LIB is None:
        path = _build.LIB if _build.LIB.exists() else _build.build()
        L = ctypes.CDLL(str(path))
        i64, f32p, vp = ctypes.c_int64, ctypes.POINTER(ctypes.c_float), ctypes.c_void_p
        L.orc_quantize_per_channel.argtypes = [vp, i64, i64, vp, vp]
        L.orc_choose_qparams.argtypes = [ctypes.c_float, ctypes.c_float, f32p, ctypes.POINTER(ctypes.c_int32)]
        L.orc_act_qparams_per_tensor.argtypes = [vp, i64, f32p, ctypes.POINTER(ctypes.c_int32)]
        L.orc_quantize_per_tensor.argtypes = [vp, i64, ctypes.c_float, ctypes.c_int32, vp]
        L.orc_quantize_per_token.argtypes = [vp, i64, i64, vp, vp]
        L.orc_gemm_u8s8.argtypes = [vp, ctypes.c_int32, vp, i64, i64, i64, vp]
        L.orc_gemm_s8s8.argtypes = [vp, vp, i64, i64, i64, vp]
        L.orc_dyn_epilogue.argtypes = [vp, i64, i64, vp, i64, vp, vp, vp]
        for f in ("orc_quantize_per_channel", "orc_choose_qparams", "orc_act_qparams_per_tensor",
                  "orc_quantize_per_tensor", "orc_quantize_per_token", "orc_gemm_u8s8",
                  "orc_gemm_s8s8", "orc_dyn_epilogue"):
            getattr(L, f).restype = None
        _LIB = L
    return _LIB


def _c(a: np.ndarray, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


# ----------------------------------------------------------------------------- weights

def quantize_per_channel(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """quant.py:25-29 in numpy: fp32 row amax clamped at 1e-8, / 127, rint (ties even), clamp ±127."""
    w = _c(w, np.float32)
    amax = np.abs(w).max(axis=1) if w.shape[1] else np.zeros(w.shape[0], np.float32)
    scale = np.maximum(amax, np.float32(1e-8)).astype(np.float32) / np.float32(127.0)
    q = np.clip(np.rint(w / scale[:, None]), -127, 127).astype(np.int8)
    return q, scale.astype(np.float32)


def quantize_per_channel_c(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Same as ``quantize_per_channel`` through the C restatement (used to cross-check both)."""
    w = _c(w, np.float32)
    n, k = w.shape
    q = np.empty((n, k), np.int8)
    s = np.empty(n, np.float32)
    lib().orc_quantize_per_channel(_p(w), n, k, _p(q), _p(s))
    return q, s


# ----------------------------------------------------------------------------- int8 (weight-only)

def int8_linear(x: np.ndarray, q: np.ndarray, scale: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """Int8Linear.forward: (x @ q^T) * scale (+ bias), dot product in float64, result fp32."""
    x2 = np.asarray(x, dtype=np.float64).reshape(-1, q.shape[1])
    y = (x2 @ q.astype(np.float64).T) * scale.astype(np.float64)
    if bias is not None:
        y = y + bias.astype(np.float64)
    return y.astype(np.float32).reshape(*np.shape(x)[:-1], q.shape[0])


def silu(v: np.ndarray) -> np.ndarray:
    v = np.asarray(v, dtype=np.float64)
    return v / (1.0 + np.exp(-v))


def gated_mlp(x, gate, up, down, h_dtype=np.float64) -> np.ndarray:
    """model.py:239-240, down(silu(gate(x)) * up(x)); each of gate/up/down is (q, scale).

    ``h_dtype`` rounds the hidden activation before the down projection, which
    lets a test state the rounding the fused GPU path applies (fp16 h).
    """
    g = np.asarray(x, np.float64).reshape(-1, gate[0].shape[1]) @ gate[0].astype(np.float64).T * gate[1]
    u = np.asarray(x, np.float64).reshape(-1, up[0].shape[1]) @ up[0].astype(np.float64).T * up[1]
    h = (silu(g) * u).astype(h_dtype).astype(np.float64)
    y = h @ down[0].astype(np.float64).T * down[1]
    return y.astype(np.float32)


# ----------------------------------------------------------------------------- int8-dyn (per tensor)

def dyn_qparams(x: np.ndarray) -> tuple[np.float32, int]:
    """Per-tensor activation scale (fp32) and zero point (0..255), fbgemm semantics."""
    x = _c(x, np.float32).reshape(-1)
    s = ctypes.c_float()
    zp = ctypes.c_int32()
    lib().orc_act_qparams_per_tensor(_p(x), x.size, ctypes.byref(s), ctypes.byref(zp))
    return np.float32(s.value), int(zp.value)


def choose_qparams(mn: float, mx: float) -> tuple[np.float32, int]:
    s = ctypes.c_float()
    zp = ctypes.c_int32()
    lib().orc_choose_qparams(float(mn), float(mx), ctypes.byref(s), ctypes.byref(zp))
    return np.float32(s.value), int(zp.value)


def dyn_quantize(x: np.ndarray, s: float, zp: int) -> np.ndarray:
    """uint8 xq = clamp(rint(fma(x, 1/s, zp)), 0, 255)."""
    x = _c(x, np.float32)
    out = np.empty(x.shape, np.uint8)
    lib().orc_quantize_per_tensor(_p(x), x.size, float(s), int(zp), _p(out))
    return out


def dyn_acc(xq: np.ndarray, zp: int, q: np.ndarray) -> np.ndarray:
    """int32 acc[m,n] = sum_k (xq[m,k] - zp) * q[n,k]."""
    xq = _c(xq, np.uint8)
    q = _c(q, np.int8)
    m, k = xq.shape
    n = q.shape[0]
    acc = np.empty((m, n), np.int32)
    lib().orc_gemm_u8s8(_p(xq), int(zp), _p(q), m, n, k, _p(acc))
    return acc


def dyn_epilogue(acc: np.ndarray, s_rows: np.ndarray, scale: np.ndarray, bias: np.ndarray | None = None) -> np.ndarray:
    """y = float(acc) * (s * scale[n]) (+ bias); ``s_rows`` is one scale or one per row."""
    acc = _c(acc, np.int32)
    m, n = acc.shape
    s_rows = _c(np.atleast_1d(s_rows), np.float32)
    stride = 0 if s_rows.size == 1 else 1
    scale = _c(scale, np.float32)
    b = None if bias is None else _c(bias, np.float32)
    y = np.empty((m, n), np.float32)
    lib().orc_dyn_epilogue(_p(acc), m, n, _p(s_rows), stride, _p(scale), None if b is None else _p(b), _p(y))
    return y


def dyn_linear(x: np.ndarray, q: np.ndarray, scale: np.ndarray, bias: np.ndarray | None = None,
               rows: np.ndarray | None = None):
    """DynamicInt8Linear.forward, bit-exact.  Returns (y, xq, s, zp, acc).

    ``rows`` restricts the GEMM and epilogue to a subset of activation rows (the
    quantisation parameters still come from the whole tensor), which keeps
    full-size checks affordable.
    """
    x2 = _c(x, np.float32).reshape(-1, q.shape[1])
    s, zp = dyn_qparams(x2)
    xsel = x2 if rows is None else x2[rows]
    xq = dyn_quantize(xsel, s, zp)
    acc = dyn_acc(xq, zp, q)
    y = dyn_epilogue(acc, np.float32(s), scale, bias)
    return y, xq, s, zp, acc


# ----------------------------------------------------------------------------- per-token mode

def tok_quantize(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-token symmetric int8: s_t = max(max|x_t|, 1e-8)/127, xq = clamp(rint(x/s_t), ±127)."""
    x = _c(x, np.float32)
    m, k = x.shape
    xq = np.empty((m, k), np.int8)
    s = np.empty(m, np.float32)
    lib().orc_quantize_per_token(_p(x), m, k, _p(xq), _p(s))
    return xq, s


def tok_linear(x: np.ndarray, q: np.ndarray, scale: np.ndarray, bias: np.ndarray | None = None):
    """Per-token int8 x int8 -> int32 GEMM with the fp32 epilogue.  Returns (y, xq, s_tok, acc)."""
    x2 = _c(x, np.float32).reshape(-1, q.shape[1])
    xq, s_tok = tok_quantize(x2)
    m, k = xq.shape
    acc = np.empty((m, q.shape[0]), np.int32)
    lib().orc_gemm_s8s8(_p(xq), _p(_c(q, np.int8)), m, q.shape[0], k, _p(acc))
    y = dyn_epilogue(acc, s_tok, scale, bias)
    return y, xq, s_tok, acc


# ----------------------------------------------------------------------------- comparators

def rel_l2(got, want) -> float:
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    den = np.linalg.norm(want)
    return float(np.linalg.norm(got - want) / (den if den > 0 else 1.0))


__all__ = [n for n in dir() if not n.startswith("_") and n not in ("annotations", "ctypes", "np", "Path")]
