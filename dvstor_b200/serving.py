"""Concurrent serving front end and the reference's breakdown reports.

The reference's compute node serves many client threads at once: each client
issues one query or one single-vector insert and waits for it, and every
operation runs its own Vamana loop with its own tiny GPU launches
(src/service/compute_service.cc:152-227; the mixed benchmark drives it from 16
client threads, tools/dvstor_breakdown_benchmark.cc:511-526).  On a B200 one
warp runs a whole query, so the server batches instead: ``BatchingServer``
collects the operations that clients have submitted, runs all pending queries
as one ``dvs_search`` call and all pending inserts as one ``dvs_insert`` call
(the two batches on the GPU at once), and hands every client its own result.
An operation's latency is its queue wait plus the batch it rode in.

``Breakdown`` records one sample per operation (enqueue, start, finish, the
GPU time of its batch) and writes the reference's breakdown JSON
(``report_to_json``, src/service/breakdown.hh:520-630): per operation the
count, the latency totals, means and p50/p95/p99 of end-to-end and service
time, the cpu/gpu/rdma/transfer split with its sub-categories, and the
counters.  RDMA and cache fields are zero: the index is in HBM.
"""
from __future__ import annotations

import threading
import time

import numpy as np

CATEGORIES = ("cpu_ns", "gpu_ns", "rdma_ns", "transfer_ns")
# the sub-categories this path can time; the reference's other names are reported as 0
SUB = {
    "query": {"gpu_ns": ("gpu_query_prepare_ns", "gpu_query_distance_ns", "gpu_query_rerank_ns"),
              "transfer_ns": ("transfer_query_h2d_ns", "transfer_distance_d2h_ns")},
    "insert": {"gpu_ns": ("gpu_insert_distance_ns", "gpu_insert_prune_ns", "gpu_insert_quantize_ns",
                          "gpu_insert_overflow_prune_ns"),
               "transfer_ns": ("transfer_insert_query_h2d_ns",)},
}
COUNTERS = ("rdma_read_bytes", "rdma_write_bytes", "neighbor_rdma_bytes", "vector_rdma_bytes", "rabitq_rdma_bytes",
            "h2d_bytes", "d2h_bytes", "l2_kernels", "prune_kernels", "rabitq_kernels", "exact_reranks",
            "visited_nodes", "visited_neighborlists", "remote_allocations", "overflow_prunes", "cache_hits",
            "cache_misses", "query_rdma_to_staging_bytes", "query_host_staging_fallback_bytes",
            "neighbor_cache_hits", "neighbor_cache_misses", "gpu_rabitq_cache_hits", "gpu_rabitq_cache_misses",
            "gpu_rabitq_cache_fills", "gpu_rabitq_cache_fill_bytes", "gpu_rabitq_cache_duplicate_fills",
            "gpu_rabitq_cache_fallback_batches", "lock_attempts", "lock_retries", "cas_failures")


def percentile_ns(values, p: float) -> int:
    """percentile_ns (src/service/breakdown.hh): the sorted value at index
    floor(p * (count - 1))."""
    if not values:
        return 0
    v = sorted(values)
    return int(v[int(p * (len(v) - 1))])


class Aggregate:
    def __init__(self, operation: str):
        self.operation = operation
        self.count = 0
        self.queue_wait = []
        self.service = []
        self.e2e = []
        self.sub = {}
        self.counters = dict.fromkeys(COUNTERS, 0)

    def add(self, queue_ns, service_ns, e2e_ns, sub_ns: dict, counters: dict):
        self.count += 1
        self.queue_wait.append(queue_ns)
        self.service.append(service_ns)
        self.e2e.append(e2e_ns)
        for k, v in sub_ns.items():
            self.sub[k] = self.sub.get(k, 0) + int(v)
        for k, v in counters.items():
            self.counters[k] += int(v)

    def category_ns(self, cat: str) -> int:
        return sum(self.sub.get(name, 0) for name in SUB[self.operation].get(cat, ()))

    def to_json(self) -> dict:
        """aggregate_to_json (src/service/breakdown.hh:520-600)."""
        n = self.count
        tq, ts, te = sum(self.queue_wait), sum(self.service), sum(self.e2e)
        gpu, rdma, xfer = self.category_ns("gpu_ns"), 0, self.category_ns("transfer_ns")
        cpu = ts - (gpu + rdma + xfer) if ts > gpu + rdma + xfer else 0
        sub = {c: {} for c in CATEGORIES}
        for cat, names in SUB[self.operation].items():
            for name in names:
                sub[cat][name] = self.sub.get(name, 0)
        sub["cpu_ns"][f"cpu_{self.operation}_runtime_overhead_ns"] = cpu
        return {
            "operation": self.operation,
            "count": n,
            "latency": {
                "queue_wait_ns": tq, "service_ns": ts, "end_to_end_ns": te,
                "mean_queue_wait_ns": tq // n if n else 0, "mean_service_ns": ts // n if n else 0,
                "mean_end_to_end_ns": te // n if n else 0,
                "p50_end_to_end_ns": percentile_ns(self.e2e, 0.50), "p95_end_to_end_ns": percentile_ns(self.e2e, 0.95),
                "p99_end_to_end_ns": percentile_ns(self.e2e, 0.99),
                "p50_service_ns": percentile_ns(self.service, 0.50), "p95_service_ns": percentile_ns(self.service, 0.95),
                "p99_service_ns": percentile_ns(self.service, 0.99),
            },
            "breakdown": {"cpu_ns": cpu, "gpu_ns": gpu, "rdma_ns": rdma, "transfer_ns": xfer},
            "sub_breakdown": sub,
            "counters": dict(self.counters),
        }

    def text_summary(self) -> str:
        """aggregate_text_summary (src/service/breakdown.hh:602-625)."""
        j = self.to_json()
        lat = j["latency"]
        ms = lambda ns: ns / 1e6  # noqa: E731
        out = [f"{self.operation} breakdown", f"  count: {self.count}",
               f"  latency_ms: mean={ms(lat['mean_end_to_end_ns']):g} p50={ms(lat['p50_end_to_end_ns']):g} "
               f"p95={ms(lat['p95_end_to_end_ns']):g} p99={ms(lat['p99_end_to_end_ns']):g}", "  top_categories:"]
        total = lat["service_ns"]
        for name, v in sorted(j["breakdown"].items(), key=lambda kv: -kv[1]):
            out.append(f"    {name}: {ms(v):g} ms ({(v / total * 100.0) if total else 0.0:g}%)")
        return "\n".join(out) + "\n"


class Breakdown:
    """Per-operation samples and the report (report_to_json, src/service/breakdown.hh:627-636)."""

    def __init__(self):
        self.lock = threading.Lock()
        self.agg = {"query": Aggregate("query"), "insert": Aggregate("insert")}

    def add(self, op, enq_ns, start_ns, end_ns, sub_ns, counters):
        with self.lock:
            self.agg[op].add(start_ns - enq_ns, end_ns - start_ns, end_ns - enq_ns, sub_ns, counters)

    def report(self, meta: dict | None = None) -> dict:
        out = {}
        for op in ("query", "insert"):
            if self.agg[op].count:
                out[f"{op}_breakdown"] = self.agg[op].to_json()
        out["bottleneck_summary"] = {op: a.text_summary() for op, a in self.agg.items() if a.count}
        out["system_counters"] = {k: sum(a.counters[k] for a in self.agg.values())
                                  for k in ("d2h_bytes", "h2d_bytes", "rdma_read_bytes", "rdma_write_bytes")}
        if meta is not None:
            out["meta"] = meta
        return out


class _Op:
    __slots__ = ("kind", "vec", "id", "enq", "done", "result", "error")

    def __init__(self, kind, vec, ident=None):
        self.kind, self.vec, self.id = kind, vec, ident
        self.enq = time.perf_counter_ns()
        self.done = threading.Event()
        self.result = self.error = None


class BatchingServer:
    """Client threads call ``search`` and ``insert`` concurrently and block until
    their own operation is done.  Two worker threads batch them: one runs every
    pending query as one ``dvs_search`` call, the other every pending insert as
    one ``dvs_insert`` call.  The library lets a search run on the GPU while an
    insert step does (inserts have their own scratch and stream), so queries
    do not wait behind an insert batch."""

    def __init__(self, index, k: int, beam_width: int, mode: str = "rabitq_gpu", beam_width_construction: int = 128,
                 alpha: float = 1.2, max_batch: int = 4096, breakdown: Breakdown | None = None):
        self.index, self.k, self.L, self.mode = index, k, beam_width, mode
        self.Lc, self.alpha, self.max_batch = beam_width_construction, alpha, max_batch
        self.breakdown = breakdown or Breakdown()
        self.cv = threading.Condition()
        self.queries, self.inserts = [], []
        self.stopping = False
        self.batches = {"query": 0, "insert": 0}
        self.workers = [threading.Thread(target=self._run, args=(kind,), name=f"dvs-{kind}", daemon=True)
                        for kind in ("query", "insert")]
        for w in self.workers:
            w.start()

    # ---- client side ----
    def search(self, query):
        """Top-k (ids, distances) of one query."""
        op = _Op("query", np.ascontiguousarray(query, np.float32).reshape(-1))
        self._submit(op)
        return op.result

    def insert(self, ident: int, vector) -> None:
        op = _Op("insert", np.ascontiguousarray(vector, np.float32).reshape(-1), int(ident))
        self._submit(op)

    def _submit(self, op):
        with self.cv:
            if self.stopping:
                raise RuntimeError("server stopped")
            (self.queries if op.kind == "query" else self.inserts).append(op)
            self.cv.notify_all()
        op.done.wait()
        if op.error is not None:
            raise op.error

    def close(self):
        with self.cv:
            self.stopping = True
            self.cv.notify_all()
        for w in self.workers:
            w.join()

    # ---- worker ----
    def _take(self, lst):
        ops = lst[:self.max_batch]
        del lst[:len(ops)]
        return ops

    def _run(self, kind):
        pending = self.queries if kind == "query" else self.inserts
        run = self._run_queries if kind == "query" else self._run_inserts
        while True:
            with self.cv:
                while not pending and not self.stopping:
                    self.cv.wait()
                if self.stopping and not pending:
                    return
                ops = self._take(pending)
            run(ops)

    def _finish(self, ops, err):
        for op in ops:
            op.error = err
            op.done.set()

    def _run_queries(self, ops):
        start = time.perf_counter_ns()
        err = None
        try:
            Q = np.stack([op.vec for op in ops])
            ids, d, st = self.index.search(Q, self.k, self.L, self.mode, stats=True)
        except Exception as e:  # every client of the batch sees the failure
            err = e
        end = time.perf_counter_ns()
        if err is None:
            gpu_ns = int(st["device_ms"] * 1e6)
            n = len(ops)
            for i, op in enumerate(ops):
                op.result = (ids[i], d[i])
                self.breakdown.add("query", op.enq, start, end,
                                   {"gpu_query_distance_ns": gpu_ns},
                                   {"h2d_bytes": Q.shape[1] * 4, "d2h_bytes": self.k * 8,
                                    "rabitq_kernels": 2 if i == 0 else 0,
                                    "exact_reranks": st["reranked"] // n, "visited_nodes": st["estimates"] // n,
                                    "visited_neighborlists": st["expansions"] // n})
            self.batches["query"] += 1
        self._finish(ops, err)

    def _run_inserts(self, ops):
        start = time.perf_counter_ns()
        err = None
        try:
            X = np.stack([op.vec for op in ops])
            ids = np.array([op.id for op in ops], np.uint32)
            st = self.index.insert(X, ids, beam_width_construction=self.Lc, alpha=self.alpha,
                                   max_batch=self.max_batch)
        except Exception as e:
            err = e
        end = time.perf_counter_ns()
        if err is None:
            n = len(ops)
            for i, op in enumerate(ops):
                self.breakdown.add("insert", op.enq, start, end,
                                   {"gpu_insert_distance_ns": int(st["device_ms"] * 1e6),
                                    "gpu_insert_prune_ns": int(st["prune_ms"] * 1e6),
                                    "gpu_insert_overflow_prune_ns": int(st["reverse_ms"] * 1e6)},
                                   {"h2d_bytes": X.shape[1] * 4 + 4, "visited_neighborlists": st["expansions"] // n,
                                    "l2_kernels": 1 if i == 0 else 0, "prune_kernels": 2 if i == 0 else 0,
                                    "overflow_prunes": st["full_prunes"] // n})
            self.batches["insert"] += 1
        self._finish(ops, err)
