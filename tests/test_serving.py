"""The concurrent serving front end (dvstor_b200.serving) on the CPU, over a
stand-in index: every client gets its own operation's result while the
server batches, failures reach every client of the batch, and the breakdown
report has the reference's layout (src/service/breakdown.hh:520-636, a report
as written by tools/dvstor_breakdown_benchmark.cc:733-747)."""
import threading
import time

import numpy as np
import pytest

from dvstor_b200.serving import BatchingServer, Breakdown, percentile_ns


class StandInIndex:
    """search returns, for query row q, ids (q[0], q[0]+1, ...) so each client can
    check it got its own answer; insert records the ids."""

    def __init__(self, fail_inserts=False):
        self.inserted = []
        self.batches = []
        self.fail_inserts = fail_inserts

    def search(self, Q, k, L, mode, stats=False):
        time.sleep(0.002)
        self.batches.append(("query", len(Q)))
        ids = (Q[:, :1].astype(np.uint32) + np.arange(k, dtype=np.uint32)[None, :])
        d = np.tile(np.arange(k, dtype=np.float32), (len(Q), 1))
        st = {"expansions": 10 * len(Q), "estimates": 100 * len(Q), "reranked": 20 * len(Q),
              "overflow_queries": 0, "device_ms": 1.5}
        return (ids, d, st) if stats else (ids, d)

    def insert(self, X, ids, beam_width_construction, alpha, max_batch):
        time.sleep(0.002)
        self.batches.append(("insert", len(X)))
        if self.fail_inserts:
            raise RuntimeError("insert failed")
        self.inserted.extend(int(i) for i in ids)
        return {"inserted": len(X), "expansions": 5 * len(X), "distances": 50 * len(X), "full_prunes": len(X),
                "device_ms": 1.0, "prune_ms": 0.5, "reverse_ms": 0.25}


def test_clients_get_their_own_results_while_batched():
    ix = StandInIndex()
    srv = BatchingServer(ix, k=5, beam_width=16)
    errors = []

    def client(c):
        for j in range(20):
            v = np.full(8, 1000 * c + j, np.float32)
            if j % 2:
                srv.insert(1_000_000 + 100 * c + j, v)
            else:
                ids, d = srv.search(v)
                if int(ids[0]) != 1000 * c + j or list(ids) != list(range(1000 * c + j, 1000 * c + j + 5)):
                    errors.append((c, j, ids))

    th = [threading.Thread(target=client, args=(c,)) for c in range(16)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    srv.close()
    assert not errors
    assert sorted(ix.inserted) == sorted(1_000_000 + 100 * c + j for c in range(16) for j in range(1, 20, 2))
    # concurrent clients were batched: fewer calls than operations
    assert len(ix.batches) < 16 * 20
    assert max(n for _, n in ix.batches) > 1


def test_batch_failure_reaches_its_clients():
    srv = BatchingServer(StandInIndex(fail_inserts=True), k=3, beam_width=8)
    with pytest.raises(RuntimeError, match="insert failed"):
        srv.insert(1, np.zeros(4, np.float32))
    ids, _ = srv.search(np.full(4, 7, np.float32))
    assert int(ids[0]) == 7
    srv.close()


def test_percentile_rule():
    # the value at floor(p * (count - 1)) of the sorted values
    v = [50, 10, 40, 20, 30]
    assert percentile_ns(v, 0.5) == 30 and percentile_ns(v, 0.99) == 40 and percentile_ns(v, 0.0) == 10
    assert percentile_ns([], 0.5) == 0


def test_breakdown_report_layout():
    bd = Breakdown()
    srv = BatchingServer(StandInIndex(), k=4, beam_width=8, breakdown=bd)
    for j in range(6):
        srv.search(np.full(8, j, np.float32))
        srv.insert(100 + j, np.zeros(8, np.float32))
    srv.close()
    rep = bd.report(meta={"client_threads": 1})
    assert set(rep) == {"bottleneck_summary", "insert_breakdown", "meta", "query_breakdown", "system_counters"}
    for op in ("query", "insert"):
        a = rep[f"{op}_breakdown"]
        assert set(a) == {"breakdown", "count", "counters", "latency", "operation", "sub_breakdown"}
        assert a["operation"] == op and a["count"] == 6
        assert set(a["breakdown"]) == {"cpu_ns", "gpu_ns", "rdma_ns", "transfer_ns"}
        lat = a["latency"]
        for key in ("queue_wait_ns", "service_ns", "end_to_end_ns", "mean_queue_wait_ns", "mean_service_ns",
                    "mean_end_to_end_ns", "p50_end_to_end_ns", "p95_end_to_end_ns", "p99_end_to_end_ns",
                    "p50_service_ns", "p95_service_ns", "p99_service_ns"):
            assert key in lat
        assert lat["end_to_end_ns"] == lat["queue_wait_ns"] + lat["service_ns"]
        assert lat["p50_end_to_end_ns"] <= lat["p99_end_to_end_ns"]
        assert a["breakdown"]["rdma_ns"] == 0
        assert f"cpu_{op}_runtime_overhead_ns" in a["sub_breakdown"]["cpu_ns"]
        assert a["counters"]["rdma_read_bytes"] == 0 and a["counters"]["h2d_bytes"] > 0
        assert rep["bottleneck_summary"][op].startswith(f"{op} breakdown\n  count: 6\n  latency_ms: mean=")
    q = rep["query_breakdown"]
    assert q["breakdown"]["gpu_ns"] == 6 * 1_500_000  # each query rode a batch with 1.5 ms of kernel time
    assert q["counters"]["visited_neighborlists"] == 6 * 10
