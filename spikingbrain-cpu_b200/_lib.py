"""ctypes binding of libsbq.so (the C ABI declared in include/sbq.h).

The library is required: importing this module raises if ``libsbq.so`` is missing, and every
status other than SBQ_OK becomes an exception (``ValueError`` for argument errors,
``RuntimeError`` for device errors), mirroring how the reference raises ``ValueError`` for bad
formats and shapes (spikingbrain_cpu/quant.py:111, loader.py:53-54).
"""

from __future__ import annotations

import ctypes
from pathlib import Path

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libsbq.so"

OK, ERR_INVALID_ARGUMENT, ERR_ALIGNMENT, ERR_UNSUPPORTED, ERR_CUDA, ERR_TIMEOUT, ERR_DEVICE, ERR_WORKSPACE = range(8)
F32, F16, BF16, I8, U8, I32 = range(6)
ACT_PER_TENSOR, ACT_PER_TOKEN = 0, 1

_c_i64, _c_int, _vp, _sz = ctypes.c_int64, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t

class GemvJob(ctypes.Structure):
    """struct sbq_gemv_job of include/sbq.h."""

    _fields_ = [("x", ctypes.c_void_p), ("ldx", ctypes.c_int64), ("packed", ctypes.c_void_p),
                ("scale", ctypes.c_void_p), ("packed_up", ctypes.c_void_p), ("scale_up", ctypes.c_void_p),
                ("bias", ctypes.c_void_p), ("n", ctypes.c_int64), ("k", ctypes.c_int64), ("y", ctypes.c_void_p),
                ("y_dtype", ctypes.c_int), ("ldy", ctypes.c_int64)]


MAX_PEERS = 8
PEER_HANDLE_BYTES = 64
PEER_SIGNAL_BYTES = 4096


class PeerGroup(ctypes.Structure):
    """struct sbq_peer_group of include/sbq.h."""

    _fields_ = [("nranks", ctypes.c_int), ("y", (ctypes.c_void_p * MAX_PEERS) * 8),
                ("signal", ctypes.c_void_p * MAX_PEERS), ("done", ctypes.c_void_p), ("wait_count", ctypes.c_void_p),
                ("wait_state", ctypes.c_void_p), ("wait_expected", ctypes.c_uint), ("wait_limit_ns", ctypes.c_ulonglong)]


# name -> (restype, argtypes); kept in the order of include/sbq.h
SIGNATURES = {
    "sbq_version": (_c_int, []),
    "sbq_last_error": (ctypes.c_char_p, []),
    "sbq_status_string": (ctypes.c_char_p, [_c_int]),
    "sbq_check_device_error": (_c_int, []),
    "sbq_packed_bytes": (_sz, [_c_i64, _c_i64]),
    "sbq_quantize_pack": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp, _vp]),
    "sbq_pack_int8": (_c_int, [_vp, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp]),
    "sbq_unpack_int8": (_c_int, [_vp, _c_i64, _c_i64, _vp, _c_i64, _vp]),
    "sbq_linear_w8": (_c_int, [_vp, _c_int, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _c_int, _c_i64, _vp]),
    "sbq_linear_w8_workspace_bytes": (_sz, [_c_i64, _c_i64, _c_int]),
    "sbq_linear_w8_ws": (_c_int, [_vp, _c_int, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _c_int, _c_i64, _vp,
                                  _sz, _vp]),
    "sbq_gemv_w8": (_c_int, [_vp, _c_int, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _c_int, _c_i64, _vp]),
    "sbq_gemm_w8a16": (_c_int, [_vp, _c_int, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _c_int, _c_i64, _vp]),
    "sbq_split_f32_bf16x2": (_c_int, [_vp, _c_i64, _c_i64, _c_i64, _vp, _vp, _c_i64, _vp]),
    "sbq_gemm_w8a16_x2": (_c_int, [_vp, _vp, _c_i64, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _c_int, _c_i64, _vp]),
    "sbq_mlp_gateup_w8": (_c_int, [_vp, _c_int, _c_i64, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _c_int,
                                   _c_i64, _vp]),
    "sbq_mlp_gateup_w8_ws": (_c_int, [_vp, _c_int, _c_i64, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _c_int,
                                      _c_i64, _vp, _sz, _vp]),
    "sbq_lora_pair_w8": (_c_int, [_vp, _c_int, _c_i64, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _c_i64, _vp, _c_int,
                                  _c_i64, _vp]),
    "sbq_gemv_w8_group": (_c_int, [ctypes.POINTER(GemvJob), _c_int, _c_int, _c_i64, _vp]),
    "sbq_gemv_w8_group_ready": (_c_int, [ctypes.POINTER(GemvJob), _c_int, _c_int, _c_int, _c_i64, _vp]),
    "sbq_gemv_plan_parts": (_c_int, [ctypes.POINTER(_c_i64), _c_int, _c_int, _c_i64, ctypes.POINTER(_c_int)]),
    "sbq_gemv_program_bytes": (_sz, [_c_int]),
    "sbq_gemv_program_sync_bytes": (_sz, [_c_int]),
    "sbq_gemv_program_build": (_c_int, [ctypes.POINTER(GemvJob), ctypes.POINTER(ctypes.c_int), _c_int, _c_int, _c_i64,
                                        _vp, _sz]),
    "sbq_gemv_program_run": (_c_int, [_vp, _c_int, _c_int, _vp, _vp]),
    "sbq_peer_alloc": (_c_int, [_sz, ctypes.POINTER(_vp)]),
    "sbq_peer_free": (_c_int, [_vp]),
    "sbq_peer_handle": (_c_int, [_vp, _vp]),
    "sbq_peer_open": (_c_int, [_vp, ctypes.POINTER(_vp)]),
    "sbq_peer_close": (_c_int, [_vp]),
    "sbq_gemv_w8_group_peer": (_c_int, [ctypes.POINTER(GemvJob), _c_int, _c_int, _c_i64, ctypes.POINTER(PeerGroup),
                                        _vp]),
    "sbq_gemv_w8_group_peer_ready": (_c_int, [ctypes.POINTER(GemvJob), _c_int, _c_int, _c_int, _c_i64,
                                              ctypes.POINTER(PeerGroup), _vp]),
    "sbq_peer_wait": (_c_int, [_vp, _vp, ctypes.c_uint, ctypes.c_ulonglong, _vp]),
    "sbq_gemv_program_build_peer": (_c_int, [ctypes.POINTER(GemvJob), ctypes.POINTER(ctypes.c_int), _c_int, _c_int,
                                             _c_i64, ctypes.POINTER(_vp), _c_int, ctypes.POINTER(_vp), _vp, _sz]),
    "sbq_dyn_workspace_bytes": (_sz, [_c_i64, _c_i64, _c_int]),
    "sbq_quant_act_per_tensor": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "sbq_quant_act_per_token": (_c_int, [_vp, _c_int, _c_i64, _c_i64, _c_i64, _vp, _vp, _vp]),
    "sbq_gemm_w8a8": (_c_int, [_vp, _c_int, _vp, _vp, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _c_i64, _vp,
                               _vp]),
    "sbq_linear_dyn": (_c_int, [_vp, _c_int, _c_i64, _c_int, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp, _c_i64,
                                _vp, _sz, _vp]),
    "sbq_linear_dyn_noalloc": (_c_int, [_vp, _c_int, _c_i64, _c_int, _vp, _vp, _vp, _vp, _c_i64, _c_i64, _c_i64, _vp,
                                        _c_i64, _vp]),
}

_LIB: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load libsbq.so once; raise if it is missing (there is no fallback path)."""
    global _LIB
    if _LIB is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                "libsbq.so is not built (%s); run the package's build.py (or __graft_entry__.build()) first" % LIB_PATH)
        lib = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


class SbqError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


class SbqArgumentError(ValueError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def check(status: int, what: str) -> None:
    if status == OK:
        return
    lib = load()
    name = lib.sbq_status_string(status).decode()
    msg = "%s failed: %s: %s" % (what, name, lib.sbq_last_error().decode())
    if status in (ERR_INVALID_ARGUMENT, ERR_ALIGNMENT, ERR_UNSUPPORTED, ERR_WORKSPACE):
        raise SbqArgumentError(status, msg)
    raise SbqError(status, msg)


def call(name: str, *args) -> None:
    """Call an int-returning entry point and raise on a non-zero status."""
    check(getattr(load(), name)(*args), name)


def packed_bytes(n: int, k: int) -> int:
    return int(load().sbq_packed_bytes(n, k))
