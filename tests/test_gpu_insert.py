"""GPU parity of the online insert (dvs_insert, Vamana::insert,
src/vamana/vamana.hh:458-999) against the oracle's restatement: after the same
inserts the device index (adjacency, records, vectors, ids, medoid) equals the
oracle's bit for bit, the per-step search counters agree, and searches of the
grown index match the oracle's knn."""
import os

import numpy as np
import pytest

from conftest import assert_results_match, normalized_gaussian, uniform_int_data, write_oracle_index

pytestmark = pytest.mark.gpu


def _stored(orc, slots):
    """Oracle slots -> stored node ids (empty slots stay empty)."""
    s = np.asarray(slots)
    return np.where(s == 0xFFFFFFFF, np.uint32(0xFFFFFFFF), orc.ids[np.minimum(s, orc.n - 1)]).astype(np.uint32)


def _assert_same_index(ix, orc):
    adj, rec, vec, ids = ix.download()
    n = orc.n
    assert ix.info.num_vectors == n and ix.info.medoid == orc.medoid
    np.testing.assert_array_equal(vec, orc.X[:n])
    np.testing.assert_array_equal(ids, orc.ids[:n])
    np.testing.assert_array_equal(rec, orc.records[:n])
    np.testing.assert_array_equal(adj, orc.adj[:n])


@pytest.mark.parametrize("R,Lc,alpha,max_batch,bits,metric,dim", [
    (16, 64, 1.2, 256, 4, "l2", 32),
    (8, 32, 1.0, 100, 4, "l2", 32),     # small R: most reverse edges meet full lists
    (24, 48, 1.2, 1, 2, "l2", 32),      # steps of one vector: the reference's sequential insert
    (16, 40, 1.2, 64, 8, "ip", 32),     # 8-bit records, IP seed distance
    (32, 128, 1.2, 256, 4, "l2", 384),  # wide rows: block-per-target reverse edges, prune in pivot passes
    (48, 64, 1.2, 128, 4, "l2", 260),   # R > 32, wide rows, dim not a multiple of 8
    (64, 96, 1.2, 128, 4, "l2", 256),   # R = 64: 65 candidates per reverse-edge prune, pair items in rounds
    (16, 200, 1.2, 64, 4, "l2", 288),   # L_c = 200 (the insert default): prune passes over 200 candidates
])
def test_insert_matches_oracle(gpu, oracle, tmp_path, R, Lc, alpha, max_batch, bits, metric, dim):
    X = normalized_gaussian(1600, dim, 41)
    n0 = 1000 if max_batch > 1 else 1400
    orc = oracle.build_index(X[:n0], R=R, L=32, bits=bits, metric=metric)
    prefix = write_oracle_index(oracle, orc, str(tmp_path / "idx"), 1)
    new = X[n0:]
    new_ids = np.arange(50_000, 50_000 + len(new), dtype=np.uint32)
    with gpu.Index(prefix) as ix:
        st = ix.insert(new, new_ids, beam_width_construction=Lc, alpha=alpha, max_batch=max_batch)
        H, E, full, steps = orc.insert(new, new_ids, beam_width_construction=Lc, alpha=alpha, max_batch=max_batch)
        assert st["inserted"] == len(new) and st["steps"] == steps
        assert st["expansions"] == H and st["distances"] == E and st["full_prunes"] == full
        _assert_same_index(ix, orc)
        if R == 8:
            assert full > 0
        Q = normalized_gaussian(120, dim, 42)
        for mode in ("rabitq_gpu", "exact_gpu"):
            ids, d = ix.search(Q, 10, 48, mode)
            o_ids, o_d, _, b_ids, b_d = orc.knn(Q, 10, 48, mode, beam_cap=48 + (64 if mode == "rabitq_gpu" else 0))
            assert_results_match(ids, d, _stored(orc, o_ids), o_d, _stored(orc, b_ids), b_d)


def test_insert_into_empty_index_grows_it(gpu, oracle):
    """dvs_create + inserts from nothing: the first vector becomes the medoid,
    steps double (1, 1, 2, 4, ...) up to max_batch; arrays grow past the initial
    capacity."""
    X = normalized_gaussian(700, 24, 43)
    P = oracle.rotation_matrix(24, 7)
    c_rot = oracle.rotate(P, oracle.centroid(X))
    tc = oracle.t_const(24, 4, 7)
    orc = oracle.OracleIndex.empty(24, 12, P, c_rot, tc, 4)
    ix = gpu.Index.create(24, 12, P, c_rot, tc, rabitq_bits=4, capacity=100)
    try:
        ids0, d0 = ix.search(X[:3], 5, 16)
        assert (ids0 == gpu.EMPTY).all() and np.isinf(d0).all()
        ix.insert(X[:1], beam_width_construction=32)
        orc.insert(X[:1], beam_width_construction=32)
        _assert_same_index(ix, orc)
        st = ix.insert(X[1:], beam_width_construction=32, max_batch=64)
        c = orc.insert(X[1:], beam_width_construction=32, max_batch=64)
        assert st["steps"] == c[3] and st["expansions"] == c[0]
        _assert_same_index(ix, orc)
        ids, d = ix.search(X[:200], 1, 32)
        assert (ids[:, 0] == np.arange(200)).mean() > 0.95
    finally:
        ix.close()


def test_service_insert_then_search(gpu, oracle, tmp_path):
    """ComputeService.insert takes (id, values) items as the reference's
    InsertItem batch (compute_service.hh:64-67, compute_service.cc:152-196)."""
    X = uniform_int_data(900, 16, 44)
    orc = oracle.build_index(X[:600], R=12, L=24)
    prefix = write_oracle_index(oracle, orc, str(tmp_path / "svc"), 2)
    svc = gpu.ComputeService(prefix, search_mode="rabitq_gpu", beam_width=32, k=5)
    assert svc.insert([(7000 + i, X[600 + i]) for i in range(300)]) == 300
    hits = [svc.search(X[600 + i], 5)[0] == 7000 + i for i in range(0, 300, 7)]
    assert np.mean(hits) > 0.9
    with pytest.raises(ValueError):
        svc.insert([(1, X[0][:5])])


def test_insert_rejects_bad_input(gpu, oracle, tmp_path):
    X = normalized_gaussian(300, 8, 45)
    orc = oracle.build_index(X, R=8, L=16)
    prefix = write_oracle_index(oracle, orc, str(tmp_path / "bad"), 1)
    with gpu.Index(prefix) as ix:
        bad = X[:2].copy()
        bad[1, 3] = np.nan
        with pytest.raises(gpu.DvsError, match="non-finite"):
            ix.insert(bad)
        with pytest.raises(gpu.DvsError, match="dimension"):
            ix.insert(np.zeros((2, 9), np.float32))
        assert ix.info.num_vectors == 300
    with gpu.Index(prefix, devices=(0, 0), placement="shard") as sh:
        with pytest.raises(gpu.DvsError, match="replicated"):
            sh.insert(X[:1])


def test_searches_run_while_inserting(gpu, oracle, tmp_path):
    """Searches from other threads while an insert runs (inserts have their own
    scratch and stream and hold the index lock only between steps): every
    search succeeds with ids of the index, and the inserts leave the device
    index equal to the oracle's, as without searches."""
    import threading

    X = normalized_gaussian(3000, 48, 46)
    orc = oracle.build_index(X[:1500], R=16, L=32)
    prefix = write_oracle_index(oracle, orc, str(tmp_path / "conc"), 1)
    Q = normalized_gaussian(200, 48, 47)
    new_ids = np.arange(90_000, 91_500, dtype=np.uint32)
    with gpu.Index(prefix) as ix:
        ix.reserve(3000)
        stop = threading.Event()
        seen = {"searches": 0, "errors": []}

        def searcher():
            while True:
                try:
                    ids, d = ix.search(Q, 10, 48)
                    ok = (ids != gpu.EMPTY) & ((ids < 1500) | ((ids >= 90_000) & (ids < 91_500)))
                    assert ok.all() and np.isfinite(d).all()
                    seen["searches"] += 1
                except Exception as e:  # reported below, in the test's thread
                    seen["errors"].append(e)
                    return
                if stop.is_set():
                    return

        th = [threading.Thread(target=searcher) for _ in range(2)]
        for t in th:
            t.start()
        try:
            ix.insert(X[1500:], new_ids, beam_width_construction=64, alpha=1.2, max_batch=100)
        finally:
            stop.set()
            for t in th:
                t.join()
        assert not seen["errors"], seen["errors"][:1]
        assert seen["searches"] > 0
        orc.insert(X[1500:], new_ids, beam_width_construction=64, alpha=1.2, max_batch=100)
        _assert_same_index(ix, orc)
