"""ctypes binding of libdvs_b200.so (declared in include/dvs_b200.h).

The library is the product: importing this module loads it and fails loudly if
it has not been built (python -m dvstor_b200.build).  There is no fallback.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from .build import LIB

DVS_OK = 0
STATUS_NAMES = {
    0: "DVS_OK", 1: "DVS_ERR_ARG", 2: "DVS_ERR_IO", 3: "DVS_ERR_FORMAT", 4: "DVS_ERR_DIM", 5: "DVS_ERR_BITS",
    6: "DVS_ERR_CUDA", 7: "DVS_ERR_PEER", 8: "DVS_ERR_HOP_LIMIT", 9: "DVS_ERR_TIMEOUT", 10: "DVS_ERR_OOM",
    11: "DVS_ERR_CAPACITY", 12: "DVS_ERR_UNSUPPORTED", 13: "DVS_ERR_NO_DEVICE",
}
MODE = {"rabitq_gpu": 0, "exact_gpu": 1}
METRIC = {"l2": 0, "ip": 1}
PLACEMENT = {"replicate": 0, "shard": 1}
EMPTY = 0xFFFFFFFF

# Every entry point declared in include/dvs_b200.h; tests check the library exports each.
EXPORTED = (
    "dvs_open", "dvs_close", "dvs_index_get_info", "dvs_index_download", "dvs_search", "dvs_search_device",
    "dvs_set_hop_limit", "dvs_set_visited_slots", "dvs_query_prepare", "dvs_rabitq_estimate", "dvs_l2_distances", "dvs_host_index_load",
    "dvs_host_index_info", "dvs_host_index_arrays", "dvs_host_index_free", "dvs_write_index", "dvs_last_error",
    "dvs_status_string", "dvs_device_count", "dvs_build_index", "dvs_set_kernel_timing", "dvs_kernel_times",
    "dvs_search_device_noalloc", "dvs_set_rotation", "dvs_query_prepare_tc", "dvs_create", "dvs_reserve",
    "dvs_insert", "dvs_index_artifacts",
)


class DvsError(RuntimeError):
    """A non-OK dvs_status, with the library's message."""

    def __init__(self, status: int, message: str):
        self.status = status
        self.name = STATUS_NAMES.get(status, f"status {status}")
        super().__init__(f"{self.name}: {message}")


class OpenParams(C.Structure):
    _fields_ = [("index_prefix", C.c_char_p), ("devices", C.POINTER(C.c_int)), ("num_devices", C.c_uint32),
                ("placement", C.c_int), ("expect_dim", C.c_uint32), ("expect_bits", C.c_uint32),
                ("expect_memory_nodes", C.c_uint32)]


class IndexInfo(C.Structure):
    _fields_ = [("num_vectors", C.c_uint64), ("dim", C.c_uint32), ("R", C.c_uint32), ("rabitq_bits", C.c_uint32),
                ("rabitq_size", C.c_uint32), ("num_memory_nodes", C.c_uint32), ("medoid", C.c_uint32),
                ("metric", C.c_int), ("t_const", C.c_double)]


class Stats(C.Structure):
    _fields_ = [("expansions", C.c_uint64), ("estimates", C.c_uint64), ("reranked", C.c_uint64),
                ("overflow_queries", C.c_uint64), ("device_ms", C.c_float)]


class WriteParams(C.Structure):
    _fields_ = [("index_prefix", C.c_char_p), ("num_vectors", C.c_uint64), ("dim", C.c_uint32), ("R", C.c_uint32),
                ("rabitq_bits", C.c_uint32), ("num_memory_nodes", C.c_uint32), ("medoid", C.c_uint32),
                ("beam_width", C.c_uint32), ("alpha", C.c_double), ("metric", C.c_int), ("t_const", C.c_double)]


class CreateParams(C.Structure):
    _fields_ = [("dim", C.c_uint32), ("R", C.c_uint32), ("rabitq_bits", C.c_uint32), ("metric", C.c_int),
                ("rotation", C.c_void_p), ("rotated_centroid", C.c_void_p), ("t_const", C.c_double),
                ("devices", C.POINTER(C.c_int)), ("num_devices", C.c_uint32), ("capacity", C.c_uint64)]


class InsertParams(C.Structure):
    _fields_ = [("beam_width_construction", C.c_uint32), ("alpha", C.c_float), ("max_batch", C.c_uint32)]


class InsertStats(C.Structure):
    _fields_ = [("inserted", C.c_uint64), ("steps", C.c_uint64), ("expansions", C.c_uint64),
                ("distances", C.c_uint64), ("full_prunes", C.c_uint64), ("device_ms", C.c_float),
                ("prune_ms", C.c_float), ("reverse_ms", C.c_float), ("max_incoming", C.c_uint32)]


_lib = None


def lib():
    """The loaded library (raises if it is missing: the CUDA path is mandatory)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            raise RuntimeError(f"{LIB} is missing; build it with `python -m dvstor_b200.build`")
        L = C.CDLL(LIB)
        vp, u32, u64, i32 = C.c_void_p, C.c_uint32, C.c_uint64, C.c_int
        sigs = {
            "dvs_open": [C.POINTER(OpenParams), C.POINTER(vp)],
            "dvs_close": [vp],
            "dvs_index_get_info": [vp, C.POINTER(IndexInfo)],
            "dvs_index_download": [vp, vp, vp, vp, vp],
            "dvs_search": [vp, vp, u32, u32, u32, u32, i32, vp, vp, C.POINTER(Stats)],
            "dvs_search_device": [vp, u32, vp, u32, u32, u32, u32, i32, vp, vp, vp, vp],
            "dvs_search_device_noalloc": [vp, u32, vp, u32, u32, u32, u32, i32, vp, vp, vp, vp],
            "dvs_set_hop_limit": [vp, u32],
            "dvs_set_visited_slots": [vp, u32],
            "dvs_set_kernel_timing": [vp, i32],
            "dvs_kernel_times": [vp, u32, C.POINTER(u32), C.POINTER(C.c_double), C.POINTER(C.c_double)],
            "dvs_query_prepare": [vp, vp, vp, vp, vp, u32, u32, u32, vp],
            "dvs_query_prepare_tc": [vp, vp, vp, vp, vp, u32, u32, u32, vp],
            "dvs_set_rotation": [vp, i32],
            "dvs_rabitq_estimate": [vp, vp, vp, vp, u32, u32, u32, vp],
            "dvs_l2_distances": [vp, vp, vp, u32, u32, vp],
            "dvs_host_index_load": [C.c_char_p, C.POINTER(vp)],
            "dvs_host_index_info": [vp, C.POINTER(IndexInfo)],
            "dvs_host_index_arrays": [vp, C.POINTER(vp), C.POINTER(vp), C.POINTER(vp), C.POINTER(vp), C.POINTER(vp),
                                      C.POINTER(vp)],
            "dvs_write_index": [C.POINTER(WriteParams), vp, vp, vp, vp, vp, vp],
            "dvs_create": [C.POINTER(CreateParams), C.POINTER(vp)],
            "dvs_reserve": [vp, u64],
            "dvs_index_artifacts": [vp, vp, vp],
            "dvs_insert": [vp, vp, vp, u32, u32, C.POINTER(InsertParams), C.POINTER(InsertStats)],
        }
        for name, args in sigs.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = C.c_int
        L.dvs_host_index_free.argtypes = [vp]
        L.dvs_host_index_free.restype = None
        L.dvs_last_error.argtypes = []
        L.dvs_last_error.restype = C.c_char_p
        L.dvs_status_string.argtypes = [i32]
        L.dvs_status_string.restype = C.c_char_p
        L.dvs_device_count.argtypes = []
        L.dvs_device_count.restype = C.c_int
        _lib = L
    return _lib


def check(status: int) -> None:
    if status != DVS_OK:
        msg = lib().dvs_last_error()
        raise DvsError(status, msg.decode() if msg else "")


def ptr(a) -> C.c_void_p | None:
    """Address of a numpy array or a torch tensor (host or device)."""
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return C.c_void_p(a.ctypes.data)
    return C.c_void_p(a.data_ptr())
