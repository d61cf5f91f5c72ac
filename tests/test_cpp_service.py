"""The C++ host side (include/dvs_b200_service.hpp: ComputeService over the C
ABI), driven through tests/cpp/service_check.cpp: the reference service's
option checks and errors on the CPU; on a GPU, search results equal to the
Python binding's (and so to the oracle's) in both modes, and insert +
store_index giving the oracle's insert bit for bit."""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT, assert_results_match, normalized_gaussian, write_oracle_index

EMPTY = 0xFFFFFFFF


def _compile(tmp_path):
    from dvstor_b200.build import LIB, build

    build()
    libdir = os.path.dirname(LIB)
    exe = str(tmp_path / "service_check")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                    os.path.join(ROOT, "tests", "cpp", "service_check.cpp"), "-L", libdir, "-ldvs_b200",
                    f"-Wl,-rpath,{libdir}", "-o", exe], check=True)
    return exe


def test_cpp_service_option_checks_and_errors(tmp_path):
    out = subprocess.run([_compile(tmp_path), "config"], check=True, capture_output=True, text=True).stdout
    got = dict(line.split(": ", 1) for line in out.strip().splitlines())
    assert got == {
        "required": "Parameters beam-width (ef-search), k, and dim are required",
        "mode": "--search-mode must be exact_gpu or rabitq_gpu",
        "bits": "--rabitq-bits must be 1, 2, 4, or 8",
        "load_store": "--store-index and --load-index cannot be used in conjunction",
        "prefix": "/data/sift/dump/index_m32_efc128",
        "beam": "beam_width must be >= k",
        "normalized": "rabitq_gpu",
        "load_missing": "failed (message)",
        "dim": "search dimension mismatch",
        "insert_dim": "insert dimension mismatch",
        "no_index": "no index loaded",
        "status": "running 0 8",
    }


@pytest.mark.gpu
def test_cpp_service_search_matches_binding_and_oracle(gpu, oracle, tmp_path):
    X = normalized_gaussian(2000, 32, 61)
    orc = oracle.build_index(X, R=16, L=32, bits=4)
    prefix = write_oracle_index(oracle, orc, str(tmp_path / "idx" / "idx"), 2)
    Q = normalized_gaussian(40, 32, 62)
    qfile = str(tmp_path / "q.f32")
    Q.tofile(qfile)
    exe = _compile(tmp_path)
    k, L = 10, 48
    for mode in ("rabitq_gpu", "exact_gpu"):
        ofile = str(tmp_path / f"out_{mode}.u32")
        subprocess.run([exe, "search", prefix, "32", str(k), str(L), mode, qfile, str(len(Q)), ofile], check=True,
                       capture_output=True, text=True)
        cpp = np.fromfile(ofile, np.uint32).reshape(2, len(Q), k)
        np.testing.assert_array_equal(cpp[0], cpp[1])  # search one by one == search_batch
        with gpu.Index(prefix) as ix:
            ids, d = ix.search(Q, k, L, mode)
        np.testing.assert_array_equal(cpp[0], ids)
        o_ids, o_d, _, b_ids, b_d = orc.knn(Q, k, L, mode, beam_cap=L + (64 if mode == "rabitq_gpu" else 0))
        assert_results_match(ids, d, o_ids, o_d, b_ids, b_d)


@pytest.mark.gpu
def test_cpp_service_insert_and_store_match_oracle(gpu, oracle, tmp_path):
    X = normalized_gaussian(1800, 32, 63)
    n0 = 1500
    orc = oracle.build_index(X[:n0], R=16, L=32, bits=4)
    prefix = write_oracle_index(oracle, orc, str(tmp_path / "base" / "idx"), 1)
    new = X[n0:]
    vfile = str(tmp_path / "v.f32")
    new.tofile(vfile)
    stored = str(tmp_path / "stored" / "idx")
    os.makedirs(os.path.dirname(stored))
    out = subprocess.run([_compile(tmp_path), "insert", prefix, "32", "10", "48", vfile, str(len(new)), "50000",
                          stored], check=True, capture_output=True, text=True).stdout
    assert out.split() == ["inserted", str(len(new)), "vectors_inserted", str(len(new)), "store", "ok"]
    new_ids = np.arange(50_000, 50_000 + len(new), dtype=np.uint32)
    orc.insert(new, new_ids, beam_width_construction=64, alpha=1.2, max_batch=1024)
    with gpu.Index(stored) as ix:
        adj, rec, vec, ids = ix.download()
        assert ix.info.num_vectors == orc.n and ix.info.medoid == orc.medoid
    np.testing.assert_array_equal(vec, orc.X[:orc.n])
    np.testing.assert_array_equal(ids, orc.ids[:orc.n])
    np.testing.assert_array_equal(rec, orc.records[:orc.n])
    np.testing.assert_array_equal(adj, orc.adj[:orc.n])
