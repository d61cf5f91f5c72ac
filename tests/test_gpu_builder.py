"""GPU offline builder (dvs_build_index) against the oracle's restatement of the
reference builder: same graph, medoid, rotation, rotated centroid, t_const and
RaBitQ records, bit for bit, and byte-identical shard files."""
import filecmp
import os

import numpy as np
import pytest

from conftest import normalized_gaussian, uniform_int_data, write_oracle_index

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,X,R,L,bits", [
    ("int", uniform_int_data(3000, 32, 1), 16, 32, 4),
    ("gauss", normalized_gaussian(4000, 48, 2), 24, 48, 4),
    ("r48", normalized_gaussian(2500, 40, 3), 48, 64, 2),
    ("ragged", normalized_gaussian(1200, 30, 4), 12, 24, 1),
])
def test_gpu_builder_matches_oracle(gpu, oracle, tmp_path, name, X, R, L, bits):
    from dvstor_b200.builder import build_index

    batch_cap = 64
    st, adj, rec = build_index(X, str(tmp_path / "gpu" / "idx"), R=R, beam_width=L, rabitq_bits=bits, seed=1234,
                               batch_cap=batch_cap, return_arrays=True)
    o_adj, o_med = oracle.build_graph(X, R, L, 1.0, 1234, batch_cap=batch_cap)
    assert st["medoid"] == o_med
    np.testing.assert_array_equal(adj, o_adj)
    d = X.shape[1]
    P = oracle.rotation_matrix(d, 1234)
    c_rot = oracle.rotate(P, oracle.centroid(X))
    tc = oracle.t_const(d, bits, 1234)
    o_rec = oracle.quantize_batch(X, P, c_rot, tc, bits)
    np.testing.assert_array_equal(rec, o_rec)
    idx = oracle.OracleIndex(X, o_adj, o_med, o_rec, P, c_rot, tc, bits)
    opre = write_oracle_index(oracle, idx, str(tmp_path / "orc" / "idx"))
    gpre = str(tmp_path / "gpu" / "idx")
    assert filecmp.cmp(opre + "_node1_of1.dat", gpre + "_node1_of1.dat", shallow=False)
    assert filecmp.cmp(opre + ".rotation.bin", gpre + ".rotation.bin", shallow=False)


def test_gpu_builder_default_schedule_and_search(gpu, oracle, tmp_path):
    """Default batch cap (2% of n); the built index opens and answers queries with
    the recall of the oracle's search on the same files."""
    from dvstor_b200.builder import build_index

    X = normalized_gaussian(6000, 64, 7)
    pre = str(tmp_path / "idx")
    st = build_index(X, pre, R=32, beam_width=64, num_memory_nodes=2)
    assert 16 < st["mean_degree"] <= 32 and st["batches"] > 5
    o_adj, o_med = oracle.build_graph(X, 32, 64, 1.0, 1234)
    info, adj, rec, vec, ids, P, c = gpu.load_host_index(pre)
    np.testing.assert_array_equal(adj, o_adj)
    Q = normalized_gaussian(200, 64, 8)
    with gpu.Index(pre) as ix:
        g_ids, g_d = ix.search(Q, 10, 64)
    idx = oracle.OracleIndex(vec, adj, info.medoid, rec, P, c, info.t_const, 4)
    o_ids, o_d, _ = idx.knn(Q, 10, 64)
    np.testing.assert_array_equal(g_d, o_d)


def test_gpu_builder_rejects_bad_arguments(gpu, tmp_path):
    from dvstor_b200.builder import build_index

    X = normalized_gaussian(100, 8, 1)
    for kw, name in [({"R": 0}, "DVS_ERR_ARG"), ({"R": 65}, "DVS_ERR_ARG"), ({"rabitq_bits": 3}, "DVS_ERR_BITS")]:
        with pytest.raises(gpu.DvsError) as e:
            build_index(X, None, **kw)
        assert e.value.name == name
    bad = X.copy()
    bad[3, 3] = np.inf
    with pytest.raises(gpu.DvsError):
        build_index(bad, None)


def test_gpu_builder_inner_product_index(gpu, oracle, tmp_path):
    """metric "ip" (the reference builder's --ip-dist) on unit-norm data: the
    same graph and records as the L2 build, the metadata says "ip", and a
    search (1 - dot medoid seed) equals the oracle's knn with the IP seed on
    the same files."""
    import json

    from dvstor_b200.builder import build_index

    X = normalized_gaussian(3000, 48, 9)
    st_l2, adj_l2, rec_l2 = build_index(X, str(tmp_path / "l2" / "idx"), R=24, beam_width=48, batch_cap=64,
                                        return_arrays=True)
    pre = str(tmp_path / "ip" / "idx")
    st_ip, adj_ip, rec_ip = build_index(X, pre, R=24, beam_width=48, batch_cap=64, return_arrays=True, metric="ip")
    np.testing.assert_array_equal(adj_ip, adj_l2)
    np.testing.assert_array_equal(rec_ip, rec_l2)
    assert json.load(open(pre + ".meta.json"))["distance"] == "ip"
    orc = oracle.read_index(pre)
    assert orc.metric == "ip"
    Q = normalized_gaussian(200, 48, 10)
    with gpu.Index(pre) as ix:
        assert ix.info.metric == 1
        ids, d = ix.search(Q, 10, 48)
    o_ids, o_d, _, b_ids, b_d = orc.knn(Q, 10, 48, beam_cap=48 + 64)
    from conftest import assert_results_match

    assert_results_match(ids, d, o_ids, o_d, b_ids, b_d)
