"""GPU parity of the whole query path (dvs_search through the C ABI) against the
oracle's restatement of Vamana::knn on the same index files and queries: final
distances bit for bit, ids bit for bit outside groups of exactly equal distance,
and the per-query work counters (expansions H, estimates E, reranked rows C_r)
exactly."""
import os

import numpy as np
import pytest

from conftest import assert_results_match, normalized_gaussian, uniform_int_data, write_oracle_index
from dvstor_b200.datasets import low_rank_uniform

pytestmark = pytest.mark.gpu


class Case:
    def __init__(self, oracle, tmp, name, X, R, Lb, bits=4, M=1, metric="l2", seed=1234):
        self.idx = oracle.build_index(X, R=R, L=Lb, bits=bits, seed=seed, metric=metric)
        self.prefix = write_oracle_index(oracle, self.idx, os.path.join(tmp, name, "idx"), M)


@pytest.fixture(scope="module")
def cases(oracle, tmp_path_factory):
    tmp = str(tmp_path_factory.mktemp("idx"))
    return {
        "int128": Case(oracle, tmp, "int128", uniform_int_data(4000, 128, 0), 32, 64),
        "gauss96": Case(oracle, tmp, "gauss96", normalized_gaussian(5000, 96, 2), 32, 64),
        "r48": Case(oracle, tmp, "r48", normalized_gaussian(3000, 64, 4), 48, 64),
        "bits2": Case(oracle, tmp, "bits2", normalized_gaussian(2000, 40, 5), 16, 32, bits=2),
        "bits1": Case(oracle, tmp, "bits1", normalized_gaussian(2000, 64, 6), 16, 32, bits=1),
        "bits8": Case(oracle, tmp, "bits8", normalized_gaussian(2000, 64, 13), 16, 32, bits=8),
        "bits8d30": Case(oracle, tmp, "bits8d30", normalized_gaussian(1500, 30, 14), 16, 32, bits=8),
        "bits8d160": Case(oracle, tmp, "bits8d160", normalized_gaussian(1200, 160, 15), 24, 32, bits=8),
        "bits2d520": Case(oracle, tmp, "bits2d520", normalized_gaussian(800, 520, 16), 16, 32, bits=2),
        "bits1d1040": Case(oracle, tmp, "bits1d1040", normalized_gaussian(600, 1040, 17), 16, 32, bits=1),
        # wide records whose dimension is not a multiple of 4: partial last words
        "d301": Case(oracle, tmp, "d301", normalized_gaussian(900, 301, 18), 24, 32),
        "bits2d490": Case(oracle, tmp, "bits2d490", normalized_gaussian(700, 490, 19), 16, 32, bits=2),
        "ragged": Case(oracle, tmp, "ragged", normalized_gaussian(1500, 30, 7), 16, 32),
        "ip": Case(oracle, tmp, "ip", normalized_gaussian(2000, 48, 8), 16, 32, metric="ip"),
        "shards": Case(oracle, tmp, "shards", uniform_int_data(3000, 32, 9), 24, 48, M=3),
        "tiny": Case(oracle, tmp, "tiny", normalized_gaussian(12, 8, 10), 4, 8),
        "d160": Case(oracle, tmp, "d160", normalized_gaussian(1500, 160, 11), 24, 32),
        "d256r48": Case(oracle, tmp, "d256r48", normalized_gaussian(1200, 256, 12), 48, 48),
        # the 1M x 960 workload's shape at small n: low-rank uniform data, R=48
        "d960r48": Case(oracle, tmp, "d960r48", low_rank_uniform(2500, 960, 4), 48, 64),
    }


def run_both(gpu, oracle, case, Q, k, L, mode="rabitq_gpu"):
    idx = case.idx
    with gpu.Index(case.prefix) as ix:
        ids, d, st = ix.search(Q, k, L, mode, stats=True)
    cap = L + 64 if mode == "rabitq_gpu" else L
    o_ids, o_d, o_cnt, b_ids, b_d = idx.knn(Q, k, L, mode, beam_cap=cap)
    return ids, d, st, o_ids, o_d, o_cnt, b_ids, b_d


@pytest.mark.parametrize("name,L", [("int128", 64), ("gauss96", 64), ("gauss96", 128), ("r48", 100), ("bits2", 32),
                                    ("bits1", 48), ("bits8", 48), ("bits8d30", 32), ("ragged", 40), ("ip", 32),
                                    ("shards", 64), ("d160", 40), ("d256r48", 48), ("d960r48", 200),
                                    ("bits8d160", 40), ("bits2d520", 32), ("bits1d1040", 32), ("d301", 40),
                                    ("bits2d490", 32)])
@pytest.mark.parametrize("mode", ["rabitq_gpu", "exact_gpu"])
def test_search_matches_oracle(gpu, oracle, cases, name, L, mode):
    case = cases[name]
    d = case.idx.dim
    if name in ("int128", "shards"):
        Q = uniform_int_data(300, d, 99)
    elif name == "d960r48":
        Q = low_rank_uniform(300, d, [4, 99])
    else:
        Q = normalized_gaussian(300, d, 99)
    k = 10
    ids, dist, st, o_ids, o_d, o_cnt, b_ids, b_d = run_both(gpu, oracle, case, Q, k, L, mode)
    assert_results_match(ids, dist, o_ids, o_d, b_ids, b_d)
    assert st["expansions"] == int(o_cnt[:, 0].sum())
    assert st["estimates"] == int(o_cnt[:, 1].sum())
    assert st["reranked"] == int(o_cnt[:, 2].sum())


@pytest.mark.parametrize("mode", ["rabitq_gpu", "exact_gpu"])
def test_k100_wide_records(gpu, oracle, cases, mode):
    """k = 100 at beam width 200 on D = 960, R = 48 (488-byte codes)."""
    case = cases["d960r48"]
    Q = low_rank_uniform(120, 960, [4, 98])
    ids, d, st, o_ids, o_d, o_cnt, b_ids, b_d = run_both(gpu, oracle, case, Q, 100, 200, mode)
    assert_results_match(ids, d, o_ids, o_d, b_ids, b_d)
    assert st["estimates"] == int(o_cnt[:, 1].sum())
    assert st["reranked"] == int(o_cnt[:, 2].sum())


def test_k_larger_than_beam_and_index(gpu, oracle, cases):
    case = cases["tiny"]
    Q = normalized_gaussian(20, 8, 3)
    ids, d, st, o_ids, o_d, o_cnt, b_ids, b_d = run_both(gpu, oracle, case, Q, 16, 16)
    assert_results_match(ids, d, o_ids, o_d, b_ids, b_d)
    for q in range(len(Q)):
        c = int(o_cnt[q, 3])
        assert c <= 12 and (ids[q, c:] == gpu.EMPTY).all() and np.isinf(d[q, c:]).all()


def test_k_equals_beam_width_exact(gpu, oracle, cases):
    case = cases["gauss96"]
    Q = normalized_gaussian(64, 96, 5)
    ids, d, st, o_ids, o_d, o_cnt, b_ids, b_d = run_both(gpu, oracle, case, Q, 32, 32, "exact_gpu")
    assert_results_match(ids, d, o_ids, o_d, b_ids, b_d)


def test_query_is_its_own_nearest_neighbour(gpu, cases):
    case = cases["gauss96"]
    with gpu.Index(case.prefix) as ix:
        ids, d = ix.search(case.idx.X[:200], 10, 64)
    assert (ids[:, 0] == np.arange(200)).mean() > 0.97


def test_repeat_runs_are_identical_and_batches_independent(gpu, cases):
    case = cases["int128"]
    Q = uniform_int_data(500, 128, 3)
    with gpu.Index(case.prefix) as ix:
        a = ix.search(Q, 10, 64)
        b = ix.search(Q, 10, 64)
        c = ix.search(Q[123:124], 10, 64)
        e = ix.search(Q[:0], 10, 64)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[0][123:124], c[0])
    assert e[0].shape == (0, 10)


def test_visited_table_hash_widths(gpu, oracle, tmp_path):
    """Indexes of 2^20 nodes or more hash visited ids with 24-bit bijections
    (a 1024-bucket minimum), smaller ones with 20-bit bijections (tables sized to
    the beam): both exact, on an index just past 2^20 nodes and on a small one."""
    from dvstor_b200.builder import build_index

    n = (1 << 20) + 4096
    X = normalized_gaussian(n, 8, 31)
    prefix = str(tmp_path / "big" / "idx")
    build_index(X, prefix, R=16, beam_width=24, device=0)
    orc = oracle.read_index(prefix)
    Q = normalized_gaussian(200, 8, 32)
    with gpu.Index(prefix) as ix:
        for mode, L in (("rabitq_gpu", 32), ("exact_gpu", 48)):
            ids, d, st = ix.search(Q, 10, L, mode, stats=True)
            o_ids, o_d, o_cnt, b_ids, b_d = orc.knn(Q, 10, L, mode, beam_cap=L + (64 if mode == "rabitq_gpu" else 0))
            assert_results_match(ids, d, o_ids, o_d, b_ids, b_d)
            assert st["estimates"] == int(o_cnt[:, 1].sum())


def test_overflow_path_is_exact(gpu, oracle, cases):
    """Queries whose visited set spills from the shared-memory table to the
    global-memory table return the same results (spill forced by shrinking the
    shared-memory table to 2 slots per beam entry)."""
    case = cases["gauss96"]
    Q = normalized_gaussian(100, 96, 21)
    with gpu.Index(case.prefix) as ix:
        ix.set_visited_slots(2)
        ids, d, st = ix.search(Q, 10, 64, stats=True)
    o_ids, o_d, o_cnt, b_ids, b_d = case.idx.knn(Q, 10, 64, beam_cap=128)
    assert st["overflow_queries"] == 100
    assert_results_match(ids, d, o_ids, o_d, b_ids, b_d)
    assert st["estimates"] == int(o_cnt[:, 1].sum())


def test_spill_table_epochs_wrap(gpu, oracle, cases):
    """A warp's spill table is not cleared between queries: each spilling query
    takes the next 8-bit epoch, and entries of other epochs count as empty.
    300 back-to-back searches give every warp slot more spilling queries than
    there are epochs, so the table is reused under every epoch and cleared at
    the wrap; every search must still equal the oracle."""
    import torch

    case = cases["gauss96"]
    Q = normalized_gaussian(64, 96, 22)
    o_ids, o_d, o_cnt, b_ids, b_d = case.idx.knn(Q, 10, 64, beam_cap=128)
    with gpu.Index(case.prefix) as ix:
        ix.set_visited_slots(2)
        dq = torch.from_numpy(Q).cuda()
        c = torch.zeros((64, 4), dtype=torch.int32, device="cuda")
        outs = []
        for _ in range(300):
            ids, d = ix.search_device(dq, 10, 64, d_counters=c)
            outs.append((ids.clone(), d.clone(), c.clone()))
        torch.cuda.synchronize()
    for ids, d, cnt in outs:
        assert_results_match(ids.cpu().numpy().view(np.uint32), d.cpu().numpy(), o_ids, o_d, b_ids, b_d)
        np.testing.assert_array_equal(cnt.cpu().numpy().view(np.uint32)[:, :3], o_cnt[:, :3])


def test_hop_limit_reports_error(gpu, cases):
    case = cases["gauss96"]
    with gpu.Index(case.prefix) as ix:
        ix.set_hop_limit(3)
        with pytest.raises(gpu.DvsError) as e:
            ix.search(normalized_gaussian(4, 96, 1), 10, 64)
        assert e.value.name == "DVS_ERR_HOP_LIMIT"
        ix.set_hop_limit(0)
        ix.search(normalized_gaussian(4, 96, 1), 10, 64)


def test_argument_errors(gpu, cases):
    case = cases["gauss96"]
    with gpu.Index(case.prefix) as ix:
        for args, name in [((normalized_gaussian(2, 95, 1), 10, 64), "DVS_ERR_DIM"),
                           ((normalized_gaussian(2, 96, 1), 10, 5), "DVS_ERR_ARG"),
                           ((normalized_gaussian(2, 96, 1), 0, 64), "DVS_ERR_ARG")]:
            with pytest.raises(gpu.DvsError) as e:
                ix.search(*args)
            assert e.value.name == name
        bad = normalized_gaussian(2, 96, 1)
        bad[1, 3] = np.nan
        with pytest.raises(gpu.DvsError, match="non-finite") as e:
            ix.search(bad, 10, 64)
        assert e.value.name == "DVS_ERR_ARG"
        # device path: the non-finite query is flagged in its counters and left
        # empty; the finite one is searched as usual
        import torch

        bad[0, 5] = np.inf
        good = normalized_gaussian(1, 96, 2)
        dq = torch.from_numpy(np.concatenate([bad, good])).cuda()
        cnt = torch.zeros((3, 4), dtype=torch.int32, device="cuda")
        ids, d = ix.search_device(dq, 10, 64, d_counters=cnt)
        torch.cuda.synchronize()
        c = cnt.cpu().numpy().view(np.uint32)
        assert ((c[:2, 3] >> 16) == 8).all() and (c[:2, :3] == 0).all()
        assert (ids[:2].cpu().numpy().view(np.uint32) == gpu.EMPTY).all() and torch.isinf(d[:2]).all()
        ref_ids, ref_d = ix.search(good, 10, 64)
        np.testing.assert_array_equal(ids[2].cpu().numpy().view(np.uint32), ref_ids[0])
    with pytest.raises(gpu.DvsError) as e:
        gpu.Index(case.prefix, expect_dim=64)
    assert e.value.name == "DVS_ERR_DIM"
    with pytest.raises(gpu.DvsError) as e:
        gpu.Index(case.prefix, expect_bits=1)
    assert e.value.name == "DVS_ERR_BITS"


def test_device_search_with_torch_buffers(gpu, oracle, cases):
    import torch

    case = cases["gauss96"]
    Q = normalized_gaussian(128, 96, 17)
    with gpu.Index(case.prefix) as ix:
        h_ids, h_d = ix.search(Q, 10, 64)
        dq = torch.from_numpy(Q).cuda()
        cnt = torch.zeros((128, 4), dtype=torch.int32, device="cuda")
        d_ids, d_d = ix.search_device(dq, 10, 64, d_counters=cnt)
        torch.cuda.synchronize()
    np.testing.assert_array_equal(d_ids.cpu().numpy().view(np.uint32), h_ids)
    np.testing.assert_array_equal(d_d.cpu().numpy(), h_d)
    _, _, o_cnt = case.idx.knn(Q, 10, 64)
    np.testing.assert_array_equal(cnt.cpu().numpy()[:, :3].astype(np.uint32), o_cnt[:, :3])


def test_index_download_matches_files(gpu, cases):
    case = cases["shards"]
    with gpu.Index(case.prefix) as ix:
        adj, rec, vec, ids = ix.download()
    np.testing.assert_array_equal(adj, case.idx.adj)
    np.testing.assert_array_equal(rec, case.idx.records)
    np.testing.assert_array_equal(vec, case.idx.X)
    np.testing.assert_array_equal(ids, np.arange(len(ids)))


def test_compute_service_single_query(gpu, cases):
    case = cases["gauss96"]
    svc = gpu.ComputeService(case.prefix, search_mode="rabitq_gpu", beam_width=64, k=10)
    out = svc.search(case.idx.X[7], 10)
    assert out[0] == 7 and len(out) == 10


def test_plumbing_workload_parity(gpu, oracle, tmp_path):
    """The CPU-runnable plumbing workload: 10,000 x 128 uniform-int vectors
    (seed 0), 1,000 queries (seed 1), R=32, build L=128, 4-bit, k=10, L=64."""
    X = uniform_int_data(10000, 128, 0)
    Q = uniform_int_data(1000, 128, 1)
    case = Case(oracle, str(tmp_path), "cfg1", X, 32, 128)
    ids, d, st, o_ids, o_d, o_cnt, b_ids, b_d = run_both(gpu, oracle, case, Q, 10, 64)
    ties = assert_results_match(ids, d, o_ids, o_d, b_ids, b_d)
    assert st["expansions"] == int(o_cnt[:, 0].sum()) and st["estimates"] == int(o_cnt[:, 1].sum())
    Xd, Qd = X.astype(np.float64), Q.astype(np.float64)
    d2 = (Qd ** 2).sum(1)[:, None] - 2 * Qd @ Xd.T + (Xd ** 2).sum(1)[None]  # exact for integer data
    gt = np.argsort(d2, 1, kind="stable")[:, :10]
    recall = np.mean([len(set(ids[i]) & set(gt[i])) / 10 for i in range(len(Q))])
    o_recall = np.mean([len(set(o_ids[i]) & set(gt[i])) / 10 for i in range(len(Q))])
    assert abs(recall - o_recall) <= ties / (10 * len(Q)) + 1e-12


@pytest.mark.parametrize("devices", [(0, 0), (0, 0, 0, 0)])
def test_sharded_layout_matches_replicated(gpu, cases, devices):
    """Sharded placement (node g in shard g mod S, the memory-node layout of
    assign_nodes_to_shards) through the shard pointer tables, all shards on
    one device: identical results and a gathered download equal to the files."""
    case = cases["shards"]
    Q = uniform_int_data(400, 32, 41)
    with gpu.Index(case.prefix) as ix:
        ref_ids, ref_d = ix.search(Q, 10, 48)
    with gpu.Index(case.prefix, devices=devices, placement="shard") as ix:
        ids, d = ix.search(Q, 10, 48)
        adj, rec, vec, stored = ix.download()
    np.testing.assert_array_equal(ids, ref_ids)
    np.testing.assert_array_equal(d.view(np.uint32), ref_d.view(np.uint32))
    np.testing.assert_array_equal(adj, case.idx.adj)
    np.testing.assert_array_equal(rec, case.idx.records)
    np.testing.assert_array_equal(vec, case.idx.X)


def test_sharded_across_gpus_reads_peer_memory(gpu, cases):
    """Two shards on two GPUs: every query reads the other GPU's shard over
    NVLink peer access; results equal the replicated index's."""
    n = gpu.lib().dvs_device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    case = cases["gauss96"]
    Q = normalized_gaussian(600, 96, 43)
    with gpu.Index(case.prefix) as ix:
        ref_ids, ref_d = ix.search(Q, 10, 64)
    with gpu.Index(case.prefix, devices=(0, 1), placement="shard") as ix:
        ids, d = ix.search(Q, 10, 64)
    np.testing.assert_array_equal(ids, ref_ids)
    np.testing.assert_array_equal(d.view(np.uint32), ref_d.view(np.uint32))


def test_sharded_rejects_bad_device_counts(gpu, cases):
    with pytest.raises(gpu.DvsError) as e:
        gpu.Index(cases["gauss96"].prefix, devices=(0, 0, 0), placement="shard")
    assert e.value.name == "DVS_ERR_ARG"


@pytest.mark.parametrize("name,L", [("gauss96", 64), ("d256r48", 48), ("d960r48", 200)])
def test_tensor_core_rotation_search(gpu, oracle, cases, name, L):
    """With the rotation on tensor cores the rest of the path is unchanged: the
    search equals the oracle's knn fed the GPU's rotated queries and factors."""
    import torch

    from dvstor_b200._lib import check, lib, ptr

    case = cases[name]
    d = case.idx.dim
    Q = normalized_gaussian(300, d, 61)
    dQ = torch.from_numpy(Q).cuda()
    dP = torch.from_numpy(case.idx.P).cuda()
    dc = torch.from_numpy(case.idx.c_rot).cuda()
    qr = torch.empty((300, d), dtype=torch.float32, device="cuda")
    fac = torch.empty((300, 3), dtype=torch.float32, device="cuda")
    check(lib().dvs_query_prepare_tc(ptr(dQ), ptr(dP), ptr(dc), ptr(qr), ptr(fac), 300, d, case.idx.bits, None))
    torch.cuda.synchronize()
    with gpu.Index(case.prefix) as ix:
        ix.set_rotation("tensor")
        ids, dist, st = ix.search(Q, 10, L, stats=True)
    o_ids, o_d, o_cnt, b_ids, b_d = case.idx.knn(Q, 10, L, q_rot=qr.cpu().numpy(), factors=fac.cpu().numpy(),
                                                 beam_cap=L + 64)
    assert_results_match(ids, dist, o_ids, o_d, b_ids, b_d)
    assert st["estimates"] == int(o_cnt[:, 1].sum())
