"""Multi-rank host logic on CPU: world_size 2 gloo ranks run ReplicaSearch with
the oracle's knn as every rank's search function (the GPU search is the same
function of the same index per rank).  Rank 0 must get exactly the
single-process answer for batches that do and do not divide evenly."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import ROOT, normalized_gaussian


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, prefix_arrays, nq_list, out_dir):
    import sys

    sys.path.insert(0, ROOT)
    import torch.distributed as dist

    from dvstor_b200.distributed import ReplicaSearch
    from oracle import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    X, Q = prefix_arrays
    idx = O.build_index(X, R=16, L=32, threads=1)
    rs = ReplicaSearch(lambda q: idx.knn(q, 10, 32, threads=1)[:2], dim=X.shape[1], k=10)
    for nq in nq_list:
        res = rs.search(Q[:nq] if rank == 0 else None)
        if rank == 0:
            np.save(os.path.join(out_dir, f"ids_{nq}.npy"), res[0])
            np.save(os.path.join(out_dir, f"d_{nq}.npy"), res[1])
    dist.barrier()
    dist.destroy_process_group()


def test_chunk_bounds_partition():
    from dvstor_b200.distributed import chunk_bounds

    for n in (0, 1, 7, 10, 1000):
        for w in (1, 2, 3, 8):
            spans = [chunk_bounds(n, w, r) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))


def test_replica_search_two_gloo_ranks(oracle, tmp_path):
    X = normalized_gaussian(1500, 24, 51)
    Q = normalized_gaussian(101, 24, 52)
    nq_list = [101, 2, 1]
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, (X, Q), nq_list, str(tmp_path))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    idx = oracle.build_index(X, R=16, L=32, threads=1)
    for nq in nq_list:
        ids, d, _ = idx.knn(Q[:nq], 10, 32)
        np.testing.assert_array_equal(np.load(tmp_path / f"ids_{nq}.npy"), ids)
        np.testing.assert_array_equal(np.load(tmp_path / f"d_{nq}.npy"), d)
