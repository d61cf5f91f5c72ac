"""The flag-compatible service front end (dvstor_b200/service.py): the
reference's flags, aliases, defaults and compute-node checks
(src/common/configuration.hh:87-205), the default index prefix
(src/common/index_path.hh:14-24), and on the GPU the service cycle
load_index -> search -> insert -> store_index -> load_index
(src/service/compute_service.cc:152-347)."""
import os

import numpy as np
import pytest

from conftest import normalized_gaussian, write_oracle_index

BASE = ["--beam-width", "32", "--k", "5", "--dim", "16"]


def test_defaults_and_aliases():
    from dvstor_b200.service import parse_config

    c = parse_config(BASE)
    assert (c.beam_width_construction, c.R, c.alpha, c.rabitq_bits, c.search_mode) == (200, 64, 1.2, 1, "exact_gpu")
    c = parse_config(["--ef-search", "40", "-k", "10", "--dim", "8", "--ef-construction", "120", "-m", "24",
                      "--search-mode", "RaBitQ_GPU", "--rabitq-bits", "4", "-t", "8", "-C", "2", "--cache",
                      "--gpu-device", "1"])
    assert (c.beam_width, c.k, c.beam_width_construction, c.R, c.threads, c.coroutines) == (40, 10, 120, 24, 8, 2)
    assert c.search_mode == "rabitq_gpu" and c.rabitq_bits == 4 and c.cache and c.gpu_device == 1


@pytest.mark.parametrize("argv,msg", [
    (["--k", "5", "--dim", "16"], "beam-width (ef-search), k, and dim are required"),
    (BASE + ["--store-index", "--load-index", "--index-prefix", "x"], "cannot be used in conjunction"),
    (BASE + ["--load-index"], "--data-path or --index-prefix is required"),
    (BASE + ["--cache", "--cache-ratio", "0"], "--cache-ratio must be > 0"),
    (BASE + ["--search-mode", "cpu"], "--search-mode must be exact_gpu or rabitq_gpu"),
    (BASE + ["--rabitq-bits", "3"], "--rabitq-bits must be 1, 2, 4, or 8"),
    (BASE + ["-t", "4", "--insert-workers", "5"], "cannot exceed --threads"),
    (BASE + ["-t", "4", "--insert-workers", "1", "--query-workers", "2"], "must equal --threads"),
    (BASE + ["-C", "2", "--query-coroutines", "3"], "cannot exceed --coroutines"),
    (["--beam-width", "4", "--k", "5", "--dim", "16"], "beam_width must be >= k"),
])
def test_rejected_flag_combinations(argv, msg):
    import re

    from dvstor_b200.service import ConfigError, parse_config

    with pytest.raises(ConfigError, match=re.escape(msg)):
        parse_config(argv)


def test_default_index_prefix():
    from dvstor_b200.service import parse_config

    c = parse_config(BASE + ["-d", "/data/sift/base.fvecs", "-m", "32", "--ef-construction", "128"])
    assert c.resolved_index_prefix() == "/data/sift/dump/index_m32_efc128"
    c = parse_config(BASE + ["-d", "/data/sift"])
    assert c.resolved_index_prefix() == "/data/sift/dump/index_m64_efc200"
    c = parse_config(BASE + ["--index-prefix", "/x/idx"])
    assert c.resolved_index_prefix() == "/x/idx"


def test_write_index_keeps_node_ids(oracle, tmp_path, dvs):
    """dvs_write_index with an ids array stores them in the node headers."""
    X = normalized_gaussian(300, 16, 70)
    idx = oracle.build_index(X, R=8, L=16)
    ids = np.arange(300, dtype=np.uint32) * 7 + 11
    prefix = str(tmp_path / "ids")
    dvs.write_index(prefix, idx.X, idx.adj, idx.records, idx.P, idx.c_rot, idx.medoid, idx.t_const, 4,
                    num_memory_nodes=2, ids=ids)
    info, adj, rec, vec, got, P, c = dvs.load_host_index(prefix)
    np.testing.assert_array_equal(got, ids)
    np.testing.assert_array_equal(adj, idx.adj)


@pytest.mark.gpu
def test_service_cycle(gpu, oracle, tmp_path):
    from dvstor_b200.service import Service

    X = normalized_gaussian(1400, 16, 71)
    idx = oracle.build_index(X[:1000], R=12, L=24, bits=4)
    prefix = write_oracle_index(oracle, idx, str(tmp_path / "svc" / "idx"), 2)
    svc = Service.from_args(BASE + ["--search-mode", "rabitq_gpu", "--rabitq-bits", "4", "--load-index",
                                    "--index-prefix", prefix, "-t", "4"])
    try:
        assert svc.status() == {"state": "running", "vectors_inserted": 0, "dimension": 16, "threads": 4}
        assert svc.search(X[3], 5)[0] == 3
        assert svc.insert([(90_000 + i, X[1000 + i]) for i in range(400)]) == 400
        assert svc.status()["vectors_inserted"] == 400
        st = svc.statistics()
        assert st["processed_inserts"] == 400 and st["processed_queries"] == 1 and st["build_distcomps"] > 0
        before = svc.search_batch(X[1000:1100], 5)
        ok, msg = svc.store_index(str(tmp_path / "stored" / "idx"), num_memory_nodes=3)
        assert ok, msg
        ok, msg = svc.load_index(str(tmp_path / "stored" / "idx"))
        assert ok, msg
        after = svc.search_batch(X[1000:1100], 5)
        np.testing.assert_array_equal(before[0], after[0])
        np.testing.assert_array_equal(before[1].view(np.uint32), after[1].view(np.uint32))
        assert (before[0][:, 0] == np.arange(90_000, 90_100)).mean() > 0.9
        ok, msg = svc.load_index(os.path.join(str(tmp_path), "missing", "idx"))
        assert not ok and msg
    finally:
        svc.close()
    bad = Service.from_args(BASE + ["--search-mode", "rabitq_gpu", "--rabitq-bits", "2", "--index-prefix", prefix])
    ok, msg = bad.load_index(prefix)
    assert not ok and "bits mismatch" in msg
