"""ctypes binding of libfp8gq.so (include/fp8gq.h).

There is no fallback: if the library cannot be loaded, every op raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from . import _build

_lock = threading.Lock()
_lib = None

STATUS = {
    0: "FP8GQ_OK",
    1: "FP8GQ_ERR_NULL_POINTER",
    2: "FP8GQ_ERR_SHAPE",
    3: "FP8GQ_ERR_ALIGNMENT",
    4: "FP8GQ_ERR_STRIDE",
    5: "FP8GQ_ERR_WORKSPACE",
    6: "FP8GQ_ERR_DEVICE",
    7: "FP8GQ_ERR_LAUNCH",
    8: "FP8GQ_ERR_UNSUPPORTED",
    9: "FP8GQ_ERR_DEVICE_TIMEOUT",
    10: "FP8GQ_ERR_SCRATCH_LIMIT",
}

MAX_GATHER_RANKS = 8   # FP8GQ_MAX_GATHER_RANKS


class Gather(ctypes.Structure):
    """struct fp8gq_gather (include/fp8gq.h)."""
    _fields_ = [("out", ctypes.c_void_p * MAX_GATHER_RANKS),
                ("flags", ctypes.c_void_p * MAX_GATHER_RANKS),
                ("counter", ctypes.c_void_p),
                ("seq", ctypes.c_void_p),
                ("ldo", ctypes.c_int64),
                ("col0", ctypes.c_int),
                ("world", ctypes.c_int),
                ("rank", ctypes.c_int),
                ("wait_input", ctypes.c_int),
                ("local_out", ctypes.c_int),
                ("tagged", ctypes.c_int)]


class ChainLinear(ctypes.Structure):
    """struct fp8gq_chain_linear (include/fp8gq.h)."""
    _fields_ = [("x", ctypes.c_void_p), ("w", ctypes.c_void_p), ("ldw", ctypes.c_int64),
                ("ws", ctypes.c_void_p), ("ldws", ctypes.c_int64), ("N", ctypes.c_int), ("K", ctypes.c_int),
                ("src", ctypes.c_int), ("swiglu", ctypes.c_int), ("col0", ctypes.c_int), ("reserved", ctypes.c_int),
                ("out", ctypes.c_void_p * MAX_GATHER_RANKS)]


class ChainPlan(ctypes.Structure):
    """struct fp8gq_chain_plan (include/fp8gq.h)."""
    _fields_ = [("device", ctypes.c_void_p), ("bytes", ctypes.c_size_t),
                ("n", ctypes.c_int), ("device_id", ctypes.c_int), ("grid", ctypes.c_int), ("stages", ctypes.c_int),
                ("world", ctypes.c_int), ("rank", ctypes.c_int), ("smem", ctypes.c_size_t),
                ("flags", ctypes.c_void_p * MAX_GATHER_RANKS), ("counter", ctypes.c_void_p),
                ("seq", ctypes.c_void_p), ("reserved", ctypes.c_int64 * 4)]


class LaunchPlan(ctypes.Structure):
    """struct fp8gq_launch_plan (include/fp8gq.h): opaque, copyable bytes."""
    _fields_ = [("opaque", ctypes.c_uint64 * 512)]


class StackLinear(ctypes.Structure):
    """struct fp8gq_stack_linear (include/fp8gq.h)."""
    _fields_ = [("x", ctypes.c_void_p), ("ldx", ctypes.c_int64),
                ("w", ctypes.c_void_p), ("ldw", ctypes.c_int64),
                ("ws", ctypes.c_void_p), ("ldws", ctypes.c_int64),
                ("out", ctypes.c_void_p), ("ldo", ctypes.c_int64),
                ("N", ctypes.c_int), ("K", ctypes.c_int),
                ("swiglu", ctypes.c_int), ("reserved", ctypes.c_int)]


class StackPlan(ctypes.Structure):
    """struct fp8gq_stack_plan (include/fp8gq.h)."""
    _fields_ = [("device", ctypes.c_void_p), ("bytes", ctypes.c_size_t),
                ("n", ctypes.c_int), ("M", ctypes.c_int), ("device_id", ctypes.c_int), ("grid", ctypes.c_int),
                ("stages", ctypes.c_int), ("npw", ctypes.c_int),
                ("sw", ctypes.c_int), ("lg_sw", ctypes.c_int), ("kpb", ctypes.c_int), ("nacc", ctypes.c_int),
                ("smem", ctypes.c_size_t), ("reserved", ctypes.c_int64 * 4)]


# name -> (restype, argtypes); the order of include/fp8gq.h
_P = ctypes.c_void_p
_I = ctypes.c_int
_I64 = ctypes.c_int64
_SZ = ctypes.c_size_t
SIGNATURES = {
    "fp8gq_version": (_I, []),
    "fp8gq_status_string": (ctypes.c_char_p, [_I]),
    "fp8gq_fused_gemv_quant": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I, _I, _I, _P, _P, _P, _SZ, _P]),
    "fp8gq_workspace_bytes": (_SZ, [_I, _I, _I]),
    "fp8gq_gemv_quant_row": (_I, [_P, _P, _I64, _P, _I64, _P, _I, _I, _P, _P, _P]),
    "fp8gq_gemv_quant_tm": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I, _I, _I, _P, _P, _P, _SZ, _P]),
    "fp8gq_fused_swiglu_q_gemm": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I, _I, _I, _P, _P, _P, _SZ, _P]),
    "fp8gq_group_quant": (_I, [_P, _I64, _I, _I, _P, _P, _P]),
    "fp8gq_swiglu_group_quant": (_I, [_P, _I64, _I, _I, _P, _P, _P]),
    "fp8gq_device_error": (_I, [ctypes.POINTER(ctypes.c_uint32), _I]),
    "fp8gq_set_wait_limit_ns": (_I, [ctypes.c_uint64, ctypes.POINTER(ctypes.c_uint64)]),
    "fp8gq_add_rmsnorm": (_I, [_P, _I64, _P, _I64, _P, ctypes.c_float, _P, _I64, _P, _I64, _I, _I, _P]),
    "fp8gq_fused_add_rmsnorm_gemv_quant": (_I, [_P, _I64, _P, _I64, _P, ctypes.c_float, _P, _I64, _P, _I64,
                                                _P, _I64, _P, _I64, _I, _I, _I, _P, _P, _P, _SZ, _P]),
    "fp8gq_fused_gemv_quant_gather": (_I, [_P, _I64, _P, _I64, _P, _I64, _I, _I, _I, ctypes.POINTER(Gather),
                                           _P, _SZ, _P]),
    "fp8gq_gather_wait": (_I, [ctypes.POINTER(Gather), _P]),
    "fp8gq_gather_decode": (_I, [ctypes.POINTER(Gather), _I, _I, _P, _I64, _P]),
    "fp8gq_fused_swiglu_q_gemm_gather": (_I, [_P, _I64, _P, _I64, _P, _I64, _I, _I, _I, ctypes.POINTER(Gather),
                                              _P, _SZ, _P]),
    "fp8gq_fused_reduce_add_rmsnorm_gemv_quant": (_I, [_P, _I, _I64, _I64, _P, _I64, _P, ctypes.c_float, _P, _I64,
                                                       _P, _I64, _P, _I64, _P, _I64, _I, _I, _I, _P, _P,
                                                       ctypes.POINTER(Gather), _P, _SZ, _P]),
    "fp8gq_ipc_get": (_I, [_P, _P, ctypes.POINTER(ctypes.c_uint64)]),
    "fp8gq_ipc_open": (_I, [_P, ctypes.c_uint64, ctypes.POINTER(_P), ctypes.POINTER(_P)]),
    "fp8gq_ipc_close": (_I, [_P]),
    "fp8gq_swiglu": (_I, [_P, _I64, _P, _I64, _P, _I64, _I, _I, _P]),
    "fp8gq_swiglu_quant": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I, _I, _P]),
    "fp8gq_set_static_weights": (_I, [_I]),
    "fp8gq_set_tm_options": (_I, [_I]),
    "fp8gq_stack_plan_bytes": (_SZ, [_I, _I]),
    "fp8gq_stack_dependencies": (_I, [ctypes.POINTER(StackLinear), _I, _I, ctypes.POINTER(_I)]),
    "fp8gq_stack_prepare": (_I, [ctypes.POINTER(StackLinear), _I, _I, _P, _SZ, ctypes.POINTER(StackPlan), _P]),
    "fp8gq_stack_run": (_I, [ctypes.POINTER(StackPlan), _P]),
    "fp8gq_chain_plan_bytes": (_SZ, [_I]),
    "fp8gq_chain_prepare": (_I, [ctypes.POINTER(ChainLinear), _I, ctypes.POINTER(Gather), _P, _SZ,
                                 ctypes.POINTER(ChainPlan)]),
    "fp8gq_chain_run": (_I, [ctypes.POINTER(ChainPlan), _P]),
    "fp8gq_gemv_quant_tm_noalloc": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I, _I, _I, _P, _P, _P]),
    "fp8gq_prepare_fused_gemv_quant": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I, _I, _I, _P, _P, _P, _SZ,
                                            ctypes.POINTER(LaunchPlan)]),
    "fp8gq_prepare_fused_swiglu_q_gemm": (_I, [_P, _I64, _P, _I64, _P, _I64, _P, _I64, _I, _I, _I, _P, _P, _P, _SZ,
                                               ctypes.POINTER(LaunchPlan)]),
    "fp8gq_prepare_fused_gemv_quant_gather": (_I, [_P, _I64, _P, _I64, _P, _I64, _I, _I, _I, ctypes.POINTER(Gather),
                                                   _P, _SZ, ctypes.POINTER(LaunchPlan)]),
    "fp8gq_prepare_fused_swiglu_q_gemm_gather": (_I, [_P, _I64, _P, _I64, _P, _I64, _I, _I, _I,
                                                      ctypes.POINTER(Gather), _P, _SZ, ctypes.POINTER(LaunchPlan)]),
    "fp8gq_prepare_fused_reduce_add_rmsnorm_gemv_quant": (_I, [_P, _I, _I64, _I64, _P, _I64, _P, ctypes.c_float, _P,
                                                               _I64, _P, _I64, _P, _I64, _P, _I64, _I, _I, _I, _P, _P,
                                                               ctypes.POINTER(Gather), _P, _SZ,
                                                               ctypes.POINTER(LaunchPlan)]),
    "fp8gq_prepare_gather_wait": (_I, [ctypes.POINTER(Gather), ctypes.POINTER(LaunchPlan)]),
    "fp8gq_prepare_gather_decode": (_I, [ctypes.POINTER(Gather), _I, _I, _P, _I64, ctypes.POINTER(LaunchPlan)]),
    "fp8gq_launch_plans": (_I, [ctypes.POINTER(LaunchPlan), _I, _P]),
}


class Fp8gqError(RuntimeError):
    """A libfp8gq entry point returned a non-zero status."""

    def __init__(self, status: int, what: str):
        self.status = status
        super().__init__(f"{what}: {STATUS.get(status, status)} ({status_string(status)})")


def library_path() -> Path:
    return _build.LIB_PATH


def load(build_if_missing: bool = True):
    """Load (building first when the .so is missing or stale and nvcc exists)."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        path = _build.LIB_PATH
        if build_if_missing and not _build.up_to_date():
            try:
                _build.build()
            except RuntimeError:
                if not path.exists():
                    raise
        if not path.exists():
            raise RuntimeError(f"{path} is missing: build it with `python -m fp8gq._build`")
        lib = ctypes.CDLL(str(path))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def status_string(status: int) -> str:
    lib = _lib
    if lib is None:
        return STATUS.get(status, "unknown")
    return lib.fp8gq_status_string(status).decode()


def check(status: int, what: str) -> None:
    if status != 0:
        raise Fp8gqError(status, what)


def set_static_weights(enable: bool) -> bool:
    """Declare that weights and block scales are never written by work queued
    earlier on the calling stream (see fp8gq_set_static_weights in
    include/fp8gq.h).  Returns the previous setting."""
    return bool(load().fp8gq_set_static_weights(1 if enable else 0))


TM_STREAM_ACTIVATIONS = 1     # FP8GQ_TM_STREAM_ACTIVATIONS
TM_WORKSPACE_SPLITK = 2       # FP8GQ_TM_WORKSPACE_SPLITK
TM_PREQUANT_ACTIVATIONS = 4   # FP8GQ_TM_PREQUANT_ACTIVATIONS
TM_RESIDENT_ACTIVATIONS = 8   # FP8GQ_TM_RESIDENT_ACTIVATIONS


def set_tm_options(flags: int) -> int:
    """Tile-kernel strategy switches, a mask of at most one activation feed
    (TM_STREAM_ACTIVATIONS, TM_PREQUANT_ACTIVATIONS, TM_RESIDENT_ACTIVATIONS)
    and TM_WORKSPACE_SPLITK (0 = pick each strategy where it fits; see
    fp8gq_set_tm_options in include/fp8gq.h).  Returns the previous mask."""
    prev = load().fp8gq_set_tm_options(int(flags))
    if prev < 0:
        raise ValueError(f"unknown or conflicting tile-kernel option bits in {flags!r}")
    return prev


def device_error(clear: bool = False) -> int:
    """Error word set by a kernel whose bounded wait gave up (0 = none)."""
    lib = load()
    code = ctypes.c_uint32(0)
    check(lib.fp8gq_device_error(ctypes.byref(code), 1 if clear else 0), "fp8gq_device_error")
    return int(code.value)


SITE_GATHER = 8   # kSiteGather: the wait for the peers' flags of a gathered call


def set_wait_limit_ns(limit_ns: int) -> int:
    """Limit of every bounded wait on the current device, in nanoseconds
    (1 ms .. 20 s; default 2 s); returns the previous limit.  Lower it only to
    make a wait run out on purpose in a test (fp8gq_set_wait_limit_ns)."""
    prev = ctypes.c_uint64(0)
    check(load().fp8gq_set_wait_limit_ns(int(limit_ns), ctypes.byref(prev)), "fp8gq_set_wait_limit_ns")
    return int(prev.value)
