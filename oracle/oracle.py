"""ctypes binding of the CPU oracle (oracle/liboracle.so).

Test and measurement infrastructure: only tests/, ``__graft_entry__.smoke()`` and
bench.py's CPU-baseline leg import this module.  The product package never does.
Each wrapper names the reference function it restates (paths relative to the
reference project root).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
EMPTY = 0xFFFFFFFF

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")
_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        u32, u64, i32, f32, f64 = C.c_uint32, C.c_uint64, C.c_int, C.c_float, C.c_double
        vp = C.c_void_p
        sig = {
            "orc_l2_ref": (f32, [_f32p, _f32p, u32]),
            "orc_seed_l2": (f32, [_f32p, _f32p, u32]),
            "orc_seed_ip": (f32, [_f32p, _f32p, u32]),
            "orc_l2_batch": (None, [_f32p, _f32p, u32, u32, _f32p]),
            "orc_rotate": (None, [_f32p, _f32p, u32, _f32p]),
            "orc_query_factors": (None, [_f32p, _f32p, u32, u32, _f32p]),
            "orc_query_prepare": (None, [_f32p, _f32p, _f32p, u32, u32, _f32p, _f32p]),
            "orc_rabitq_estimate": (None, [_f32p, _f32p, _u8p, u32, u32, u32, u32, _f32p]),
            "orc_best_rescale_factor": (f64, [_f32p, C.c_size_t, C.c_size_t]),
            "orc_t_const": (f64, [C.c_size_t, C.c_size_t, u64]),
            "orc_gaussian_matrix": (None, [u32, i32, _f64p]),
            "orc_rotation_matrix": (None, [u32, i32, _f32p]),
            "orc_centroid": (None, [_f32p, C.c_size_t, u32, _f32p]),
            "orc_quantize_rotated": (None, [_f32p, _f32p, f64, u32, u32, _u8p]),
            "orc_quantize_batch": (None, [_f32p, C.c_size_t, u32, u32, _f32p, _f32p, f64, _u8p, u32, i32]),
            "orc_compute_medoid": (u64, [_f32p, u64, u32]),
            "orc_random_init": (None, [u64, u32, u64, _u32p]),
            "orc_insert_order": (None, [u64, u64, _u32p]),
            "orc_build_beam_search": (u32, [_f32p, u64, u32, _u32p, u32, u32, _f32p, u32, _f32p, _u32p, u32]),
            "orc_robust_prune": (u32, [_f32p, u32, u32, _f32p, _u32p, u32, f32, u32, _u32p]),
            "orc_batch_schedule": (None, [u64, u64, vp, C.POINTER(u64)]),
            "orc_build_graph": (u64, [_f32p, u64, u32, u32, u32, f32, u64, u64, i32, _u32p]),
            "orc_write_shards": (i32, [C.c_char_p, _f32p, u64, u32, u32, u32, _u32p, u32, _u8p, _f32p, _f32p,
                                       f64, u32, u32, f64, i32]),
            "orc_knn": (i32, [u32, u32, u32, u32, u32, u32, _u32p, _u8p, u32, _f32p, _f32p, _f32p, _f32p, u32,
                              u32, u32, i32, vp, vp, _u32p, _f32p, _u32p, vp, vp, u32, i32]),
            "orc_make_deterministic_vector": (None, [u32, u64, _f32p]),
            "orc_quantize_gpu_rotated": (None, [_f32p, _f32p, f64, u32, u32, _u8p]),
            "orc_robust_prune_gpu": (u32, [_f32p, _f32p, vp, u32, u32, f32, u32, _u32p]),
            "orc_insert_batch": (i32, [C.POINTER(u32), u32, u32, u32, u32, u32, C.POINTER(u32), _u32p, _u8p, u32,
                                       _f32p, _u32p, _f32p, _f32p, f64, _f32p, _u32p, u32, u32, f32, _u64p, i32]),
            "orc_cpu_beam_search_batch": (i32, [_f32p, u64, u32, _u32p, u32, u32, _f32p, u32, u32, u32, i32,
                                                _u32p, vp]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


def rabitq_size(dim: int, bits: int) -> int:
    """VamanaNode::RABITQ_SIZE (src/vamana/vamana_node.hh:49-56)."""
    return (bits * dim + 7) // 8 + 8


def l2_ref(q, x) -> float:
    q, x = _f32(q), _f32(x)
    return float(lib().orc_l2_ref(q, x, q.size))


def l2_batch(q, cand):
    q, cand = _f32(q), _f32(cand)
    n, d = cand.shape
    out = np.empty(n, np.float32)
    lib().orc_l2_batch(q, cand, n, d, out)
    return out


def seed_dist(q, x, metric: str = "l2") -> float:
    q, x = _f32(q), _f32(x)
    f = lib().orc_seed_ip if metric == "ip" else lib().orc_seed_l2
    return float(f(q, x, q.size))


def rotate(P, x):
    P, x = _f32(P), _f32(x)
    out = np.empty(x.size, np.float32)
    lib().orc_rotate(P, x, x.size, out)
    return out


def query_factors(q_rot, c_rot, bits):
    q_rot, c_rot = _f32(q_rot), _f32(c_rot)
    f = np.empty(3, np.float32)
    lib().orc_query_factors(q_rot, c_rot, q_rot.size, bits, f)
    return f


def query_prepare(q, P, c_rot, bits):
    q = _f32(q)
    qr = np.empty(q.size, np.float32)
    f = np.empty(3, np.float32)
    lib().orc_query_prepare(q, _f32(P), _f32(c_rot), q.size, bits, qr, f)
    return qr, f


def rabitq_estimate(q_rot, f3, records, dim, bits, rec_stride=None):
    records = np.ascontiguousarray(records, dtype=np.uint8)
    n = records.shape[0]
    stride = rec_stride or records.shape[1]
    out = np.empty(n, np.float32)
    lib().orc_rabitq_estimate(_f32(q_rot), _f32(f3), records.reshape(-1), stride, n, dim, bits, out)
    return out


def best_rescale_factor(abs_unit, bits) -> float:
    a = _f32(abs_unit)
    return float(lib().orc_best_rescale_factor(a, a.size, bits))


def t_const(dim, bits, seed) -> float:
    """get_const_scaling_factors (tools/vamana_offline_builder.cc:949-973)."""
    return float(lib().orc_t_const(dim, bits, seed & 0xFFFFFFFFFFFFFFFF))


def gaussian_matrix(dim, seed):
    out = np.empty(dim * dim, np.float64)
    lib().orc_gaussian_matrix(dim, seed, out)
    return out.reshape(dim, dim).T  # (i, j) indexing of a column-major buffer


def rotation_matrix(dim, seed):
    """Column-major P, returned as a flat float32 array of dim*dim."""
    P = np.empty(dim * dim, np.float32)
    lib().orc_rotation_matrix(dim, seed, P)
    return P


def centroid(X):
    X = _f32(X)
    out = np.empty(X.shape[1], np.float32)
    lib().orc_centroid(X, X.shape[0], X.shape[1], out)
    return out


def quantize_batch(X, P, c_rot, tc, bits, threads=0):
    X = _f32(X)
    n, d = X.shape
    rs = rabitq_size(d, bits)
    out = np.zeros((n, rs), np.uint8)
    lib().orc_quantize_batch(X, n, d, bits, _f32(P), _f32(c_rot), tc, out.reshape(-1), rs, threads)
    return out


def quantize_rotated(x_rot, c_rot, tc, bits):
    x_rot = _f32(x_rot)
    out = np.zeros(rabitq_size(x_rot.size, bits), np.uint8)
    lib().orc_quantize_rotated(x_rot, _f32(c_rot), tc, x_rot.size, bits, out)
    return out


def compute_medoid(X) -> int:
    X = _f32(X)
    return int(lib().orc_compute_medoid(X, X.shape[0], X.shape[1]))


def random_init(n, R, seed):
    adj = np.empty(n * R, np.uint32)
    lib().orc_random_init(n, R, seed, adj)
    return adj.reshape(n, R)


def insert_order(n, seed):
    o = np.empty(n, np.uint32)
    lib().orc_insert_order(n, seed, o)
    return o


def batch_schedule(n, cap):
    cnt = C.c_uint64()
    lib().orc_batch_schedule(n, cap, None, C.byref(cnt))
    out = np.empty(cnt.value, np.uint64)
    lib().orc_batch_schedule(n, cap, _ptr(out), C.byref(cnt))
    return out


def build_beam_search(X, adj, medoid, q, L, cap=1 << 20):
    X, q = _f32(X), _f32(q)
    adj = np.ascontiguousarray(adj, dtype=np.uint32)
    n, d = X.shape
    od = np.empty(cap, np.float32)
    oi = np.empty(cap, np.uint32)
    m = lib().orc_build_beam_search(X, n, d, adj.reshape(-1), adj.shape[1], medoid, q, L, od, oi, cap)
    m = min(m, cap)
    return od[:m], oi[:m]


def robust_prune(X, source, cand_d, cand_id, alpha, R):
    X = _f32(X)
    out = np.empty(R, np.uint32)
    m = lib().orc_robust_prune(X, X.shape[1], source, _f32(cand_d), np.ascontiguousarray(cand_id, np.uint32),
                               len(cand_id), alpha, R, out)
    return out[:m]


def build_graph(X, R, L, alpha=1.0, seed=1234, batch_cap=None, threads=0):
    """Batched, deterministic restatement of build_vamana_graph.  Returns (adj, medoid)."""
    X = _f32(X)
    n, d = X.shape
    cap = batch_cap if batch_cap is not None else default_batch_cap(n)
    adj = np.empty(n * R, np.uint32)
    med = lib().orc_build_graph(X, n, d, R, L, alpha, seed & 0xFFFFFFFFFFFFFFFF, cap, threads, adj)
    return adj.reshape(n, R), int(med)


def default_batch_cap(n: int) -> int:
    """Largest batch of the doubling schedule: 2% of the dataset, at least 1."""
    return max(1, min(65536, (n * 2) // 100))


def write_shards(prefix, X, adj, medoid, records, P, c_rot, tc, bits, num_memory_nodes=1, beam_width=128,
                 alpha=1.2, metric="l2"):
    X = _f32(X)
    adj = np.ascontiguousarray(adj, np.uint32)
    n, d = X.shape
    rc = lib().orc_write_shards(prefix.encode(), X, n, d, adj.shape[1], bits, adj.reshape(-1), medoid,
                                np.ascontiguousarray(records, np.uint8).reshape(-1), _f32(P), _f32(c_rot), tc,
                                num_memory_nodes, beam_width, alpha, 1 if metric == "ip" else 0)
    if rc != 0:
        raise OSError(f"orc_write_shards failed for {prefix}")


def quantize_gpu_rotated(x_rot, c_rot, tc, bits):
    """rabitq_quantize_single_kernel<4,B> (src/gpu/kernels/distance_kernels.cuh:376-464)
    on a rotated vector: the online insert's quantizer."""
    x_rot = _f32(x_rot)
    out = np.empty(rabitq_size(x_rot.shape[0], bits), np.uint8)
    lib().orc_quantize_gpu_rotated(x_rot, _f32(c_rot), float(tc), x_rot.shape[0], bits, out)
    return out


def robust_prune_gpu(cand_vecs, sorted_dists, alpha, R, order=None):
    """robust_prune_kernel (src/gpu/kernels/distance_kernels.cuh:285-370): kept
    original candidate indices, in selection order."""
    V = _f32(cand_vecs)
    n, d = V.shape
    out = np.empty(max(R, 1), np.uint32)
    o = None if order is None else np.ascontiguousarray(order, np.uint32)
    cnt = lib().orc_robust_prune_gpu(V, _f32(sorted_dists), _ptr(o), n, d, np.float32(alpha), R, out)
    return out[:cnt].copy()


class OracleIndex:
    """SoA view of an index as the oracle reads it."""

    def __init__(self, X, adj, medoid, records, P, c_rot, t_const, bits, metric="l2", ids=None):
        self.X = _f32(X)
        self.adj = np.ascontiguousarray(adj, np.uint32)
        self.medoid = int(medoid)
        self.records = np.ascontiguousarray(records, np.uint8)
        self.P = _f32(P)
        self.c_rot = _f32(c_rot)
        self.t_const = float(t_const)
        self.bits = int(bits)
        self.metric = metric
        self.n, self.dim = self.X.shape
        self.R = self.adj.shape[1]
        self.ids = np.arange(self.n, dtype=np.uint32) if ids is None else np.ascontiguousarray(ids, np.uint32)

    @classmethod
    def empty(cls, dim, R, P, c_rot, t_const, bits, metric="l2"):
        return cls(np.zeros((0, dim), np.float32), np.zeros((0, R), np.uint32), 0,
                   np.zeros((0, rabitq_size(dim, bits)), np.uint8), P, c_rot, t_const, bits, metric)

    def insert(self, X, ids=None, beam_width_construction=200, alpha=1.2, max_batch=1024, threads=0):
        """Vamana::insert (src/vamana/vamana.hh:458-999) in steps of
        min(max_batch, node count) vectors: every vector of a step searches the
        graph as of the step's start, reverse edges in insert order.  Returns
        (expansions, distances, full prunes, steps)."""
        X = _f32(X).reshape(-1, self.dim)
        ids = (np.arange(self.n, self.n + X.shape[0], dtype=np.uint32) if ids is None
               else np.ascontiguousarray(ids, np.uint32))
        tot = [0, 0, 0, 0]
        pos = 0
        while pos < X.shape[0]:
            b = min(max_batch, max(self.n, 1), X.shape[0] - pos)
            c = self.insert_step(X[pos:pos + b], ids[pos:pos + b], beam_width_construction, alpha, threads)
            tot = [t + x for t, x in zip(tot, c + (1,))]
            pos += b
        return tuple(tot)

    def insert_step(self, X, ids, beam_width_construction, alpha, threads=0):
        """One step: orc_insert_batch."""
        X = _f32(X).reshape(-1, self.dim)
        B = X.shape[0]
        new_ids = np.ascontiguousarray(ids, np.uint32)
        cap = self.n + B
        pad = lambda a, rows, fill: np.concatenate([a, np.full((rows,) + a.shape[1:], fill, a.dtype)])
        self.X = pad(self.X, B, 0)
        self.adj = pad(self.adj, B, EMPTY)
        self.records = pad(self.records, B, 0)
        self.ids = pad(self.ids, B, 0)
        n = C.c_uint32(self.n)
        med = C.c_uint32(self.medoid)
        counts = np.zeros(3, np.uint64)
        rc = lib().orc_insert_batch(C.byref(n), cap, self.dim, self.R, self.bits, 1 if self.metric == "ip" else 0,
                                    C.byref(med), self.adj.reshape(-1), self.records.reshape(-1),
                                    self.records.shape[1], self.X, self.ids, self.P, self.c_rot, self.t_const, X,
                                    new_ids, B, beam_width_construction, np.float32(alpha), counts, threads)
        if rc != 0:
            raise ValueError("oracle insert rejected its arguments")
        self.n = n.value
        self.medoid = med.value
        return tuple(int(c) for c in counts)

    def knn(self, queries, k, beam_width, mode="rabitq_gpu", q_rot=None, factors=None, beam_cap=0, threads=0):
        """Vamana::knn (src/vamana/vamana.hh:57-452) over a batch of queries.

        Returns ids (nq,k), dists (nq,k), counters (nq,4: H, E, C_r, count) and,
        when beam_cap > 0, the full final beam (ids, dists)."""
        Q = _f32(queries).reshape(-1, self.dim)
        nq = Q.shape[0]
        ids = np.empty((nq, k), np.uint32)
        dists = np.empty((nq, k), np.float32)
        cnt = np.empty((nq, 4), np.uint32)
        bi = np.empty((nq, max(beam_cap, 1)), np.uint32)
        bd = np.empty((nq, max(beam_cap, 1)), np.float32)
        qr = None if q_rot is None else _f32(q_rot).reshape(nq, self.dim)
        fa = None if factors is None else _f32(factors).reshape(nq, 3)
        rc = lib().orc_knn(self.n, self.dim, self.R, self.bits, 1 if self.metric == "ip" else 0, self.medoid,
                           self.adj.reshape(-1), self.records.reshape(-1), self.records.shape[1],
                           self.X, self.P, self.c_rot, Q, nq, k, beam_width, 0 if mode == "rabitq_gpu" else 1,
                           _ptr(qr), _ptr(fa), ids, dists, cnt,
                           _ptr(bi) if beam_cap else None, _ptr(bd) if beam_cap else None, beam_cap, threads)
        if rc != 0:
            raise ValueError("oracle knn rejected its arguments (beam_width < k or k == 0)")
        if beam_cap:
            return ids, dists, cnt, bi, bd
        return ids, dists, cnt


def cpu_beam_search_batch(X, adj, medoid, queries, L, k, threads=0):
    """The reference's CPU beam_search (tools/vamana_offline_builder.cc:523-625) over a batch."""
    X = _f32(X)
    adj = np.ascontiguousarray(adj, np.uint32)
    Q = _f32(queries).reshape(-1, X.shape[1])
    nq = Q.shape[0]
    ids = np.empty((nq, k), np.uint32)
    vis = np.empty(nq, np.uint32)
    lib().orc_cpu_beam_search_batch(X, X.shape[0], X.shape[1], adj.reshape(-1), adj.shape[1], medoid, Q, nq, L, k,
                                    threads, ids, _ptr(vis))
    return ids, vis


def make_deterministic_vector(seed: int, dim: int):
    """make_deterministic_vector (test/src/main.cpp:37-51)."""
    out = np.empty(dim, np.float32)
    lib().orc_make_deterministic_vector(seed, dim, out)
    return out


def build_index(X, R=32, L=128, bits=4, seed=1234, batch_cap=None, threads=0, metric="l2"):
    """Everything the offline builder produces, restated: graph, P, c', t_const, records."""
    X = _f32(X)
    adj, med = build_graph(X, R, L, 1.0, seed, batch_cap, threads)
    d = X.shape[1]
    P = rotation_matrix(d, seed)
    c = centroid(X)
    c_rot = rotate(P, c)
    tc = t_const(d, bits, seed)
    rec = quantize_batch(X, P, c_rot, tc, bits, threads)
    return OracleIndex(X, adj, med, rec, P, c_rot, tc, bits, metric)


def read_index(prefix: str) -> OracleIndex:
    """Reads the offline files with numpy alone (meta.json, rotation.bin and the
    shards of write_vamana_shards, tools/vamana_offline_builder.cc:1136-1267)
    into the oracle's dense layout (slot g = k*M + s)."""
    import json

    meta = json.load(open(prefix + ".meta.json"))
    d, R, bits, M = int(meta["dim"]), int(meta["R"]), int(meta["rabitq_bits"]), int(meta["num_memory_nodes"])
    rs = rabitq_size(d, bits)
    node = 16 + 4 * d + rs + 8 * R
    aligned = (node + 7) & ~7
    rot = np.fromfile(prefix + ".rotation.bin", np.uint8)
    P = rot[4:4 + 4 * d * d].view(np.float32).copy()
    c_rot = rot[4 + 4 * d * d:4 + 4 * d * d + 4 * d].view(np.float32).copy()
    tc = float(rot[4 + 4 * d * d + 4 * d:4 + 4 * d * d + 4 * d + 8].view(np.float64)[0])
    shards = [np.fromfile(f"{prefix}_node{s + 1}_of{M}.dat", np.uint8) for s in range(M)]
    counts = [(int(sh[:8].view(np.uint64)[0]) - 16) // aligned for sh in shards]
    n = sum(counts)
    X = np.empty((n, d), np.float32)
    rec = np.empty((n, rs), np.uint8)
    adj = np.full((n, R), EMPTY, np.uint32)
    for s, sh in enumerate(shards):
        body = sh[16:16 + counts[s] * aligned].reshape(counts[s], aligned)
        g = np.arange(counts[s]) * M + s
        X[g] = body[:, 16:16 + 4 * d].copy().view(np.float32)
        rec[g] = body[:, 16 + 4 * d:16 + 4 * d + rs]
        ec = body[:, 12].astype(np.int64)
        ptrs = body[:, 16 + 4 * d + rs:16 + 4 * d + rs + 8 * R].copy().view(np.uint64)
        shard = (ptrs >> np.uint64(48)).astype(np.int64)
        off = (ptrs & np.uint64((1 << 48) - 1)).astype(np.int64)
        slot = (off - 16) // aligned * M + shard
        valid = (np.arange(R)[None, :] < ec[:, None]) & (ptrs != 0)
        order = np.argsort(~valid, axis=1, kind="stable")  # non-null entries first, in order
        vals = np.where(valid, slot, EMPTY).astype(np.uint32)
        adj[g] = np.take_along_axis(vals, order, axis=1)
    mp = int(shards[0][8:16].view(np.uint64)[0])
    medoid = ((mp & ((1 << 48) - 1)) - 16) // aligned * M + (mp >> 48)
    return OracleIndex(X, adj, medoid, rec, P, c_rot, tc, bits, meta.get("distance", "l2"))
