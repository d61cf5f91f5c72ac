"""GPU offline builder (dvs_build_index): graph, RaBitQ records, shard files."""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib
from ._lib import check, lib, ptr


class BuildParams(C.Structure):
    _fields_ = [("output_prefix", C.c_char_p), ("R", C.c_uint32), ("beam_width", C.c_uint32), ("alpha", C.c_double),
                ("rabitq_bits", C.c_uint32), ("seed", C.c_int32), ("num_memory_nodes", C.c_uint32),
                ("metric", C.c_int), ("device", C.c_int), ("batch_cap", C.c_uint32), ("visited_cap", C.c_uint32),
                ("out_adj", C.c_void_p), ("out_records", C.c_void_p)]


class BuildStats(C.Structure):
    _fields_ = [("medoid", C.c_uint32), ("batches", C.c_uint64), ("graph_ms", C.c_float), ("mean_visited", C.c_double),
                ("mean_degree", C.c_double)]


def build_index(X, prefix: str | None, R: int = 32, beam_width: int = 128, alpha: float = 1.2, rabitq_bits: int = 4,
                seed: int = 1234, num_memory_nodes: int = 1, device: int = 0, batch_cap: int = 0,
                visited_cap: int = 0, return_arrays: bool = False, metric: str = "l2"):
    """Builds an index from X (n, dim) float32 on `device`; writes the offline
    files at `prefix` when given.  Returns a stats dict (plus adj and records
    when return_arrays).  metric "ip" marks the index inner-product (the
    search seeds with 1 - dot); the graph is built with L2 distances, which on
    unit-norm vectors rank exactly as inner product does."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    n, d = X.shape
    adj = np.empty((n, R), np.uint32) if return_arrays else None
    rec = np.empty((n, (rabitq_bits * d + 7) // 8 + 8), np.uint8) if return_arrays else None
    if prefix:
        os.makedirs(os.path.dirname(os.path.abspath(prefix)), exist_ok=True)
    p = BuildParams(prefix.encode() if prefix else None, R, beam_width, alpha, rabitq_bits, seed, num_memory_nodes,
                    _lib.METRIC[metric], device, batch_cap, visited_cap, ptr(adj), ptr(rec))
    st = BuildStats()
    L = lib()
    fn = L.dvs_build_index
    fn.argtypes = [C.POINTER(BuildParams), C.c_void_p, C.c_uint64, C.c_uint32, C.POINTER(BuildStats)]
    fn.restype = C.c_int
    check(fn(C.byref(p), ptr(X), n, d, C.byref(st)))
    out = {"medoid": st.medoid, "batches": st.batches, "graph_ms": st.graph_ms, "mean_visited": st.mean_visited,
           "mean_degree": st.mean_degree}
    if return_arrays:
        return out, adj, rec
    return out
