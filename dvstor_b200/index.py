"""Host-side mirror of the reference's query interface over the C ABI.

``ComputeService`` keeps the reference's service knobs — ``search-mode``,
``beam-width``, ``k``, ``gpu-device`` and ``index-prefix``
(src/common/configuration.hh:83-130) — and its calls: ``search(query, k)``
returns the top-k node ids of one query (ComputeService::search,
src/service/compute_service.hh:91) and ``load_index(prefix)`` opens the offline
shard/meta/rotation files (src/service/compute_service.cc:520-593).  Batched
variants (``search_batch``) are the form the GPU is built for.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import _lib
from ._lib import DvsError, check, lib, ptr

SEARCH_MODES = ("exact_gpu", "rabitq_gpu")  # validated as at src/common/configuration.hh:170-174
RABITQ_BITS = (1, 2, 4, 8)                   # src/common/configuration.hh:176-180


class Index:
    """An index opened on one or more devices (``dvs_open``)."""

    def __init__(self, prefix: str, devices=(0,), placement: str = "replicate", expect_dim: int = 0,
                 expect_bits: int = 0, expect_memory_nodes: int = 0):
        L = lib()
        devs = (C.c_int * len(devices))(*devices)
        p = _lib.OpenParams(str(prefix).encode(), devs, len(devices), _lib.PLACEMENT[placement], expect_dim,
                            expect_bits, expect_memory_nodes)
        h = C.c_void_p()
        check(L.dvs_open(C.byref(p), C.byref(h)))
        self._h = h
        self.devices = tuple(devices)
        info = _lib.IndexInfo()
        check(L.dvs_index_get_info(self._h, C.byref(info)))
        self.info = info
        self.dim = info.dim

    @classmethod
    def create(cls, dim: int, R: int, rotation, rotated_centroid, t_const: float, rabitq_bits: int = 4,
               metric: str = "l2", devices=(0,), capacity: int = 0) -> "Index":
        """An empty index on `devices` (``dvs_create``) that inserts grow; the
        first insert becomes the medoid (src/vamana/vamana.hh:479-546)."""
        P = np.ascontiguousarray(rotation, np.float32).reshape(-1)
        c = np.ascontiguousarray(rotated_centroid, np.float32).reshape(-1)
        if P.size != dim * dim or c.size != dim:
            raise ValueError("rotation must be dim*dim and the rotated centroid dim floats")
        devs = (C.c_int * len(devices))(*devices)
        p = _lib.CreateParams(dim, R, rabitq_bits, _lib.METRIC[metric], ptr(P), ptr(c), float(t_const), devs,
                              len(devices), capacity)
        h = C.c_void_p()
        check(lib().dvs_create(C.byref(p), C.byref(h)))
        self = cls.__new__(cls)
        self._h = h
        self.devices = tuple(devices)
        self.refresh_info()
        return self

    def refresh_info(self) -> None:
        info = _lib.IndexInfo()
        check(lib().dvs_index_get_info(self._h, C.byref(info)))
        self.info = info
        self.dim = info.dim

    def reserve(self, capacity: int) -> None:
        check(lib().dvs_reserve(self._h, capacity))

    def insert(self, vectors, ids=None, beam_width_construction: int = 200, alpha: float = 1.2,
               max_batch: int = 1024) -> dict:
        """dvs_insert: Vamana::insert (src/vamana/vamana.hh:458-999) for a batch,
        in steps of min(max_batch, node count) vectors that each search the graph
        of the step's start.  Returns the insert statistics."""
        X = np.ascontiguousarray(vectors, dtype=np.float32)
        if X.ndim == 1:
            X = X[None]
        n = X.shape[0]
        idp = None
        if ids is not None:
            idp = np.ascontiguousarray(ids, dtype=np.uint32)
            if idp.shape != (n,):
                raise ValueError("ids must have one entry per vector")
        prm = _lib.InsertParams(beam_width_construction, alpha, max_batch)
        st = _lib.InsertStats()
        check(lib().dvs_insert(self._h, ptr(X), ptr(idp) if idp is not None else None, n, X.shape[1], C.byref(prm),
                               C.byref(st)))
        self.refresh_info()
        return {f: getattr(st, f) for f, _ in _lib.InsertStats._fields_}

    def close(self) -> None:
        if getattr(self, "_h", None):
            lib().dvs_close(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def set_hop_limit(self, max_expansions: int) -> None:
        check(lib().dvs_set_hop_limit(self._h, max_expansions))

    def set_rotation(self, rotation: str) -> None:
        """'exact' (fp32 FMA chains, the default) or 'tensor' (tcgen05, 3xTF32)."""
        check(lib().dvs_set_rotation(self._h, {"exact": 0, "tensor": 1}[rotation]))

    def set_kernel_timing(self, enable: bool) -> None:
        check(lib().dvs_set_kernel_timing(self._h, 1 if enable else 0))

    def kernel_times(self, device_slot: int = 0):
        """(searches, prepare_ms_sum, search_ms_sum) recorded since the last call."""
        n, pm, sm = C.c_uint32(), C.c_double(), C.c_double()
        check(lib().dvs_kernel_times(self._h, device_slot, C.byref(n), C.byref(pm), C.byref(sm)))
        return n.value, pm.value, sm.value

    def set_visited_slots(self, slots_per_beam_entry: int) -> None:
        check(lib().dvs_set_visited_slots(self._h, slots_per_beam_entry))

    def search(self, queries, k: int, beam_width: int, mode: str = "rabitq_gpu", stats: bool = False):
        """dvs_search on host arrays: returns (ids (nq,k) uint32, dists (nq,k) float32[, stats dict])."""
        if mode not in SEARCH_MODES:
            raise ValueError("search-mode must be exact_gpu or rabitq_gpu")
        Q = np.ascontiguousarray(queries, dtype=np.float32)
        if Q.ndim == 1:
            Q = Q[None]
        nq = Q.shape[0]
        ids = np.empty((nq, k), np.uint32)
        dists = np.empty((nq, k), np.float32)
        st = _lib.Stats()
        check(lib().dvs_search(self._h, ptr(Q), nq, Q.shape[1], k, beam_width, _lib.MODE[mode], ptr(ids), ptr(dists),
                               C.byref(st)))
        if stats:
            return ids, dists, {"expansions": st.expansions, "estimates": st.estimates, "reranked": st.reranked,
                                "overflow_queries": st.overflow_queries, "device_ms": st.device_ms}
        return ids, dists

    def search_device(self, d_queries, k: int, beam_width: int, mode: str = "rabitq_gpu", d_out_ids=None,
                      d_out_dist=None, d_counters=None, stream=None, device_slot: int = 0):
        """dvs_search_device on torch CUDA tensors (asynchronous on `stream`)."""
        import torch

        nq = d_queries.shape[0]
        dev = d_queries.device
        if d_out_ids is None:
            d_out_ids = torch.empty((nq, k), dtype=torch.int32, device=dev)
        if d_out_dist is None:
            d_out_dist = torch.empty((nq, k), dtype=torch.float32, device=dev)
        handle = stream.cuda_stream if stream is not None else torch.cuda.current_stream(dev).cuda_stream
        # torch's default stream has handle 0, which the C ABI reads as "the
        # library's internal stream"; pass the legacy default stream instead so
        # the search is ordered with the caller's work on it
        s = C.c_void_p(handle if handle else 1)  # 1 = cudaStreamLegacy
        check(lib().dvs_search_device(self._h, device_slot, ptr(d_queries), nq, d_queries.shape[1], k, beam_width,
                                      _lib.MODE[mode], ptr(d_out_ids), ptr(d_out_dist), ptr(d_counters), s))
        return d_out_ids, d_out_dist

    def artifacts(self):
        """(rotation P as loaded — dim*dim column-major, flattened —, rotated centroid)."""
        d = self.info.dim
        P = np.empty(d * d, np.float32)
        c = np.empty(d, np.float32)
        check(lib().dvs_index_artifacts(self._h, ptr(P), ptr(c)))
        return P, c

    def download(self):
        """Device layout back on the host: adj (n,R), records (n,rabitq_size), vecs (n,dim), ids (n,)."""
        n, i = self.info.num_vectors, self.info
        adj = np.empty((n, i.R), np.uint32)
        rec = np.empty((n, i.rabitq_size), np.uint8)
        vec = np.empty((n, i.dim), np.float32)
        ids = np.empty(n, np.uint32)
        check(lib().dvs_index_download(self._h, ptr(adj), ptr(rec), ptr(vec), ptr(ids)))
        return adj, rec, vec, ids


class ComputeService:
    """Query-side mirror of ComputeService<Distance> (src/service/compute_service.hh:84-97)."""

    def __init__(self, index_prefix: str | None = None, search_mode: str = "rabitq_gpu", beam_width: int = 128,
                 k: int = 10, gpu_device: int = 0, rabitq_bits: int | None = None, dim: int | None = None,
                 devices=None):
        if search_mode not in SEARCH_MODES:
            raise ValueError("--search-mode must be exact_gpu or rabitq_gpu")
        if rabitq_bits is not None and rabitq_bits not in RABITQ_BITS:
            raise ValueError("--rabitq-bits must be 1, 2, 4, or 8")
        if beam_width == 0 or k == 0:
            raise ValueError("Parameters beam-width (ef-search) and k are required")
        if beam_width < k:
            raise ValueError("beam_width must be >= k")  # src/vamana/vamana.hh:49
        self.search_mode = search_mode
        self.beam_width = beam_width
        self.k = k
        self.rabitq_bits = rabitq_bits
        self.dim = dim
        self.devices = tuple(devices) if devices else (gpu_device,)
        self.index: Index | None = None
        if index_prefix:
            self.load_index(index_prefix)

    def load_index(self, path: str) -> bool:
        if self.index is not None:
            self.index.close()
        self.index = Index(path, devices=self.devices, expect_dim=self.dim or 0, expect_bits=self.rabitq_bits or 0)
        self.dim = self.index.dim
        return True

    def search(self, query, k: int):
        """Top-k node ids of one query (the service truncates to k, compute_service.cc:215-217)."""
        ids, _ = self.search_batch(np.asarray(query, np.float32)[None], k)
        row = ids[0]
        return [int(x) for x in row if x != _lib.EMPTY][:k]

    def insert(self, batch, beam_width_construction: int = 200, alpha: float = 1.2) -> int:
        """ComputeService::insert (src/service/compute_service.cc:152-196): `batch`
        is a list of (id, values); returns the number inserted."""
        if self.index is None:
            raise DvsError(1, "no index loaded")
        if not batch:
            return 0
        for _, values in batch:
            if len(values) != self.dim:
                raise ValueError("insert dimension mismatch")
        ids = np.array([int(i) for i, _ in batch], np.uint32)
        X = np.array([np.asarray(v, np.float32) for _, v in batch], np.float32)
        st = self.index.insert(X, ids, beam_width_construction=beam_width_construction, alpha=alpha)
        return int(st["inserted"])

    def search_batch(self, queries, k: int | None = None):
        if self.index is None:
            raise DvsError(1, "no index loaded")
        q = np.asarray(queries, dtype=np.float32)
        if q.ndim != 2 or q.shape[1] != self.dim:
            raise ValueError("search dimension mismatch")
        kk = min(k or self.k, self.k)
        return self.index.search(q, kk, self.beam_width, self.search_mode)


def load_host_index(prefix: str):
    """Reads the offline files on the host (no GPU): (info, adj, records, vecs, ids, P, c_rot)."""
    L = lib()
    h = C.c_void_p()
    check(L.dvs_host_index_load(str(prefix).encode(), C.byref(h)))
    try:
        info = _lib.IndexInfo()
        check(L.dvs_host_index_info(h, C.byref(info)))
        pa = [C.c_void_p() for _ in range(6)]
        check(L.dvs_host_index_arrays(h, *[C.byref(x) for x in pa]))
        n, d, R, rs = info.num_vectors, info.dim, info.R, info.rabitq_size

        def arr(p, ctype, count, shape, dtype):
            buf = (ctype * count).from_address(p.value)
            return np.ctypeslib.as_array(buf).reshape(shape).astype(dtype, copy=True)

        adj = arr(pa[0], C.c_uint32, n * R, (n, R), np.uint32)
        rec = arr(pa[1], C.c_uint8, n * rs, (n, rs), np.uint8)
        vec = arr(pa[2], C.c_float, n * d, (n, d), np.float32)
        ids = arr(pa[3], C.c_uint32, n, (n,), np.uint32)
        P = arr(pa[4], C.c_float, d * d, (d * d,), np.float32)
        c = arr(pa[5], C.c_float, d, (d,), np.float32)
        return info, adj, rec, vec, ids, P, c
    finally:
        L.dvs_host_index_free(h)


def write_index(prefix: str, vecs, adj, records, rotation, rotated_centroid, medoid: int, t_const: float, bits: int,
                num_memory_nodes: int = 1, beam_width: int = 128, alpha: float = 1.2, metric: str = "l2",
                ids=None) -> None:
    """dvs_write_index: the reference's shard/meta/rotation formats (node ids:
    `ids`, or the slot numbers when None)."""
    vecs = np.ascontiguousarray(vecs, np.float32)
    adj = np.ascontiguousarray(adj, np.uint32)
    records = np.ascontiguousarray(records, np.uint8)
    P = np.ascontiguousarray(rotation, np.float32)
    c = np.ascontiguousarray(rotated_centroid, np.float32)
    n, d = vecs.shape
    os.makedirs(os.path.dirname(os.path.abspath(prefix)), exist_ok=True)
    p = _lib.WriteParams(str(prefix).encode(), n, d, adj.shape[1], bits, num_memory_nodes, medoid, beam_width, alpha,
                         _lib.METRIC[metric], t_const)
    idp = None if ids is None else np.ascontiguousarray(ids, np.uint32)
    if idp is not None and idp.shape != (n,):
        raise ValueError("ids must have one entry per vector")
    check(lib().dvs_write_index(C.byref(p), ptr(vecs), ptr(adj), ptr(records), ptr(P), ptr(c),
                                ptr(idp) if idp is not None else None))
