"""ctypes binding of libpyflame_cuda.so (include/pyflame_cuda.h).

The library is built in-tree (`python -m pyflame_b200.build`).  Loading it
needs no GPU; executing needs an sm_100 device.  There is no CPU fallback: if
the library is missing, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "lib" / "libpyflame_cuda.so"

PFC_OK = 0
ERRORS = {
    -1: "invalid argument", -2: "unsupported", -3: "CUDA error", -4: "out of memory", -5: "no device",
    -6: "graph error", -7: "JIT error", -8: "device timeout", -9: "internal error",
}


class PfcError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{ERRORS.get(code, code)}: {msg}")
        self.code = code


class DeviceInfo(C.Structure):
    _fields_ = [("device_id", C.c_int), ("name", C.c_char * 256), ("architecture", C.c_char * 32),
                ("total_memory", C.c_size_t), ("free_memory", C.c_size_t), ("compute_units", C.c_int),
                ("max_threads_per_block", C.c_int), ("warp_size", C.c_int)]


class ExecutorConfigC(C.Structure):
    _fields_ = [("device_id", C.c_int), ("enable_profiling", C.c_int), ("sync_after_launch", C.c_int),
                ("workspace_size_mb", C.c_size_t), ("precision", C.c_int), ("use_cuda_graph", C.c_int),
                ("fail_after_n_allocations", C.c_int)]


class ExecutionResultC(C.Structure):
    _fields_ = [("success", C.c_int), ("error_message", C.c_char * 1024), ("compile_time_ms", C.c_double),
                ("transfer_time_ms", C.c_double), ("compute_time_ms", C.c_double), ("total_time_ms", C.c_double),
                ("kernel_launches", C.c_int64), ("h2d_bytes", C.c_uint64), ("d2h_bytes", C.c_uint64)]


class MemoryStatsC(C.Structure):
    _fields_ = [("total_allocated", C.c_size_t), ("peak_allocated", C.c_size_t),
                ("total_allocations", C.c_size_t), ("total_deallocations", C.c_size_t),
                ("cache_hits", C.c_size_t), ("cache_misses", C.c_size_t), ("resident_constant_bytes", C.c_size_t)]


class GemmEpilogueC(C.Structure):
    _fields_ = [("alpha", C.c_float), ("bias", C.c_void_p), ("act", C.c_int), ("residual", C.c_void_p),
                ("res_sb", C.c_int64), ("res_sm", C.c_int64), ("res_sn", C.c_int64)]


class PoolParamsC(C.Structure):
    _fields_ = [(n, C.c_int64 if n != "mode" else C.c_int) for n in (
        "mode", "n", "c", "h", "w", "sn", "sc", "sh", "sw", "kh", "kw", "stride_h", "stride_w", "pad_h", "pad_w",
        "oh", "ow", "osn", "osc", "osh", "osw")]


_P = C.c_void_p
_I64 = C.c_int64
# name -> (restype, argtypes); the list is the C-ABI of include/pyflame_cuda.h
SIGNATURES = {
    "pfc_cuda_is_available": (C.c_int, []),
    "pfc_cuda_get_device_count": (C.c_int, [C.POINTER(C.c_int)]),
    "pfc_cuda_get_device_info": (C.c_int, [C.c_int, C.POINTER(DeviceInfo)]),
    "pfc_cuda_set_device": (C.c_int, [C.c_int]),
    "pfc_cuda_get_device": (C.c_int, [C.POINTER(C.c_int)]),
    "pfc_cuda_synchronize": (C.c_int, []),
    "pfc_last_error": (C.c_char_p, []),
    "pfc_abi_version": (C.c_int, []),
    "pfc_graph_create": (C.c_int, [C.POINTER(_P)]),
    "pfc_graph_destroy": (C.c_int, [_P]),
    "pfc_graph_add_node": (C.c_int, [_P, C.c_uint64, C.c_int, C.c_int, C.c_int, C.c_int, C.POINTER(_I64), C.c_int,
                                     C.POINTER(C.c_uint64)]),
    "pfc_graph_set_attr": (C.c_int, [_P, C.c_uint64, C.c_char_p, C.c_int, _P, _I64]),
    "pfc_graph_set_constant": (C.c_int, [_P, C.c_uint64, _P, C.c_size_t, C.c_uint32, C.c_uint64]),
    "pfc_graph_mark_output": (C.c_int, [_P, C.c_uint64]),
    "pfc_graph_num_nodes": (C.c_int, [_P, C.POINTER(_I64)]),
    "pfc_executor_config_default": (None, [C.POINTER(ExecutorConfigC)]),
    "pfc_executor_create": (C.c_int, [C.POINTER(ExecutorConfigC), C.POINTER(_P)]),
    "pfc_executor_destroy": (C.c_int, [_P]),
    "pfc_executor_execute": (C.c_int, [_P, _P, C.POINTER(C.c_uint64), C.c_int, C.POINTER(_P),
                                       C.POINTER(C.c_size_t), C.POINTER(ExecutionResultC)]),
    "pfc_executor_execute_device": (C.c_int, [_P, _P, C.POINTER(C.c_uint64), C.c_int, C.POINTER(_P),
                                              C.POINTER(C.c_uint64), C.c_int, C.POINTER(_P), _P,
                                              C.POINTER(ExecutionResultC)]),
    "pfc_executor_execute_streamed": (C.c_int, [_P, _P, C.POINTER(C.c_uint64), C.c_int, C.POINTER(_P),
                                                C.POINTER(C.c_uint64), C.c_int, C.POINTER(_P), C.c_int,
                                                C.POINTER(ExecutionResultC)]),
    "pfc_executor_get_device_info": (C.c_int, [_P, C.POINTER(DeviceInfo)]),
    "pfc_executor_get_memory_stats": (C.c_int, [_P, C.POINTER(MemoryStatsC)]),
    "pfc_executor_release_constants": (C.c_int, [_P]),
    "pfc_executor_set_resident": (C.c_int, [_P, C.c_uint64, _P, C.c_size_t]),
    "pfc_executor_describe_plan": (C.c_int, [_P, _P, C.POINTER(C.c_uint64), C.c_int, C.c_char_p, C.c_size_t]),
    "pfc_compile_check": (C.c_int, [_P, C.POINTER(C.c_uint64), C.c_int, C.c_int, C.c_char_p, C.c_size_t]),
    "pfc_executor_last_profile": (C.c_int, [_P, _P, C.POINTER(C.c_double), C.c_int, C.POINTER(C.c_int)]),
    "pfk_split_tf32": (C.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _P, _I64, _P]),
    "pfk_convert_bf16": (C.c_int, [_P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I64, _P]),
    "pfk_gemm": (C.c_int, [C.c_int, _P, _P, _I64, _P, _P, _I64, _I64, _I64, _I64, _I64, _I64, _P, _I64, _I64, _I64,
                           C.POINTER(GemmEpilogueC), _P, _P]),
    "pfk_im2col": (C.c_int, [_P] + [_I64] * 18 + [_P, _P, _P, _I64, _P]),
    "pfk_pool2d": (C.c_int, [_P, _P, C.POINTER(PoolParamsC), _P]),
    "pfk_matmul_tf32x3_static": (C.c_int, [_P, _P, _P, _I64, _I64, _I64, _P, _P]),
    "pfk_check_bounded_wait": (C.c_int, [_P, _I64, _P]),
}

_lib = None


def lib():
    """Load the native library (once).  Raises if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m pyflame_b200.build`")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def check(rc: int):
    if rc != PFC_OK:
        msg = lib().pfc_last_error().decode(errors="replace")
        raise PfcError(rc, msg)
    return rc


def loaded_path() -> str:
    return os.fspath(LIB_PATH)
