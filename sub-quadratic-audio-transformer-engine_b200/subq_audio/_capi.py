"""ctypes binding of the C ABI in include/kernels.hpp (libsubq_b200.so).

This is the binding a Python caller of the reference's kernel layer adds to
reach the B200 scan: plain pointers, sizes and a stream handle, no torch
types. The structures mirror the header field for field.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libsubq_b200.so")

SUBQ_OK = 0
SUBQ_ERR_INVALID_ARGUMENT = 1
SUBQ_ERR_ALIAS = 2
SUBQ_ERR_UNSUPPORTED = 3
SUBQ_ERR_CUDA = 4
SUBQ_ERR_TIMEOUT = 5
SUBQ_ERR_WORKSPACE = 6
SUBQ_ERR_STATE = 7

SUBQ_FP32, SUBQ_FP16, SUBQ_BF16, SUBQ_FP64 = 0, 1, 2, 3
SUBQ_DECAY_NONE, SUBQ_DECAY_SCALAR, SUBQ_DECAY_PER_HEAD, SUBQ_DECAY_PER_TOKEN = 0, 1, 2, 3
SUBQ_PATH_AUTO, SUBQ_PATH_EXACT, SUBQ_PATH_TENSORCORE, SUBQ_PATH_CHUNKED = 0, 1, 2, 3

# Every symbol include/kernels.hpp declares.
EXPORTED = (
    "subq_fwd", "subq_bwd", "subq_fwd_workspace_bytes", "subq_bwd_workspace_bytes",
    "subq_feature_map", "subq_last_path", "subq_last_launches", "subq_last_error",
    "subq_abi_version", "subq_device_info", "subq_device_status", "subq_bwd_noalloc",
    "subq_segment_states_bytes", "subq_selftest_wait_timeout",
    "subq_head_rmsnorm_fwd", "subq_head_rmsnorm_bwd", "subq_head_rmsnorm_bwd_workspace_bytes",
)


class Tensor4(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("stride_b", ctypes.c_int64),
                ("stride_h", ctypes.c_int64), ("stride_n", ctypes.c_int64)]


class ScanDesc(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64), ("heads", ctypes.c_int64), ("seq_len", ctypes.c_int64),
        ("head_dim", ctypes.c_int64), ("value_dim", ctypes.c_int64),
        ("dtype", ctypes.c_int32), ("normalize", ctypes.c_int32),
        ("scale", ctypes.c_float), ("clamp_min", ctypes.c_float),
        ("decay_mode", ctypes.c_int32), ("log_gamma_scalar", ctypes.c_float),
        ("log_gamma", ctypes.c_void_p), ("mask", ctypes.c_void_p), ("mask_stride_b", ctypes.c_int64),
        ("flush_subnormal", ctypes.c_int32), ("path", ctypes.c_int32),
        ("kv_heads", ctypes.c_int64), ("reverse", ctypes.c_int32),
    ]


class FwdArgs(ctypes.Structure):
    _fields_ = [
        ("desc", ScanDesc), ("q", Tensor4), ("k", Tensor4), ("v", Tensor4), ("o", Tensor4),
        ("state_in", ctypes.c_void_p), ("norm_in", ctypes.c_void_p),
        ("state_out", ctypes.c_void_p), ("norm_out", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("stream", ctypes.c_void_p), ("segment_states", ctypes.c_void_p),
    ]


class BwdArgs(ctypes.Structure):
    _fields_ = [
        ("desc", ScanDesc), ("q", Tensor4), ("k", Tensor4), ("v", Tensor4), ("dout", Tensor4),
        ("dq", Tensor4), ("dk", Tensor4), ("dv", Tensor4),
        ("state_in", ctypes.c_void_p), ("norm_in", ctypes.c_void_p),
        ("dlog_gamma", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("stream", ctypes.c_void_p), ("segment_states", ctypes.c_void_p),
        ("out", Tensor4),
    ]


class RmsArgs(ctypes.Structure):
    _fields_ = [
        ("batch", ctypes.c_int64), ("heads", ctypes.c_int64), ("seq_len", ctypes.c_int64),
        ("head_dim", ctypes.c_int64), ("dtype", ctypes.c_int32), ("eps", ctypes.c_float),
        ("x", Tensor4), ("y", Tensor4), ("dy", Tensor4), ("dx", Tensor4),
        ("weight", ctypes.c_void_p), ("dweight", ctypes.c_void_p),
        ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("stream", ctypes.c_void_p),
    ]


class SubqError(RuntimeError):
    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    """Load libsubq_b200.so, building it first if it is missing."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                import importlib.util

                spec = importlib.util.spec_from_file_location(
                    "_subq_build", os.path.join(os.path.dirname(_HERE), "build.py"))
                mod = importlib.util.module_from_spec(spec)
                spec.loader.exec_module(mod)
                mod.build_lib()
            lib = ctypes.CDLL(LIB_PATH)
            lib.subq_fwd.argtypes = [ctypes.POINTER(FwdArgs)]
            lib.subq_fwd.restype = ctypes.c_int
            lib.subq_bwd.argtypes = [ctypes.POINTER(BwdArgs)]
            lib.subq_bwd.restype = ctypes.c_int
            lib.subq_bwd_noalloc.argtypes = [ctypes.POINTER(BwdArgs)]
            lib.subq_bwd_noalloc.restype = ctypes.c_int
            lib.subq_fwd_workspace_bytes.argtypes = [ctypes.POINTER(FwdArgs)]
            lib.subq_fwd_workspace_bytes.restype = ctypes.c_size_t
            lib.subq_bwd_workspace_bytes.argtypes = [ctypes.POINTER(BwdArgs)]
            lib.subq_bwd_workspace_bytes.restype = ctypes.c_size_t
            lib.subq_segment_states_bytes.argtypes = [ctypes.POINTER(FwdArgs)]
            lib.subq_segment_states_bytes.restype = ctypes.c_size_t
            lib.subq_feature_map.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p]
            lib.subq_feature_map.restype = ctypes.c_int
            lib.subq_last_path.restype = ctypes.c_int
            lib.subq_last_launches.restype = ctypes.c_int
            lib.subq_last_error.restype = ctypes.c_char_p
            lib.subq_abi_version.restype = ctypes.c_int
            lib.subq_device_info.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t,
                                             ctypes.POINTER(ctypes.c_size_t), ctypes.POINTER(ctypes.c_int)]
            lib.subq_device_info.restype = ctypes.c_int
            lib.subq_device_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
            lib.subq_device_status.restype = ctypes.c_int
            lib.subq_selftest_wait_timeout.argtypes = [ctypes.c_int, ctypes.c_void_p]
            lib.subq_selftest_wait_timeout.restype = ctypes.c_int
            for name in ("subq_head_rmsnorm_fwd", "subq_head_rmsnorm_bwd"):
                getattr(lib, name).argtypes = [ctypes.POINTER(RmsArgs)]
                getattr(lib, name).restype = ctypes.c_int
            lib.subq_head_rmsnorm_bwd_workspace_bytes.argtypes = [ctypes.POINTER(RmsArgs)]
            lib.subq_head_rmsnorm_bwd_workspace_bytes.restype = ctypes.c_size_t
            _lib = lib
    return _lib


def check(rc: int) -> None:
    if rc != SUBQ_OK:
        msg = load().subq_last_error().decode(errors="replace")
        if rc in (SUBQ_ERR_INVALID_ARGUMENT, SUBQ_ERR_ALIAS):
            raise ValueError(msg)
        raise SubqError(rc, msg)


def fwd(args: FwdArgs) -> None:
    check(load().subq_fwd(ctypes.byref(args)))


def bwd(args: BwdArgs) -> None:
    check(load().subq_bwd(ctypes.byref(args)))


def bwd_noalloc(args: BwdArgs) -> None:
    """subq_bwd_noalloc: the backward with the library's static scratch."""
    check(load().subq_bwd_noalloc(ctypes.byref(args)))


def head_rmsnorm_fwd(args: RmsArgs) -> None:
    check(load().subq_head_rmsnorm_fwd(ctypes.byref(args)))


def head_rmsnorm_bwd(args: RmsArgs) -> None:
    check(load().subq_head_rmsnorm_bwd(ctypes.byref(args)))


def head_rmsnorm_bwd_workspace_bytes(args: RmsArgs) -> int:
    return int(load().subq_head_rmsnorm_bwd_workspace_bytes(ctypes.byref(args)))


def fwd_workspace_bytes(args: FwdArgs) -> int:
    return int(load().subq_fwd_workspace_bytes(ctypes.byref(args)))


def bwd_workspace_bytes(args: BwdArgs) -> int:
    return int(load().subq_bwd_workspace_bytes(ctypes.byref(args)))


def segment_states_bytes(args: FwdArgs) -> int:
    return int(load().subq_segment_states_bytes(ctypes.byref(args)))


def device_status(stream: int = 0) -> int:
    """Synchronises `stream` and returns (and clears) the device status word."""
    st = ctypes.c_int(0)
    check(load().subq_device_status(ctypes.c_void_p(stream), ctypes.byref(st)))
    return int(st.value)


def selftest_wait_timeout(polls: int = 1000, stream: int = 0) -> None:
    """subq_selftest_wait_timeout: a bounded device-side wait that runs out."""
    check(load().subq_selftest_wait_timeout(int(polls), ctypes.c_void_p(stream)))


def last_path() -> int:
    return int(load().subq_last_path())


def last_launches() -> int:
    return int(load().subq_last_launches())
