"""bench.py's contract pieces that need no GPU: defaults, the metric name, the
algorithmic-bytes formula of the roofline and the profile-traffic selection."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402


def _args(*argv):
    old = sys.argv
    sys.argv = ["bench.py", *argv]
    try:
        return bench.parse_args()
    finally:
        sys.argv = old


def test_defaults_are_the_headline_run():
    a = _args()
    assert a.gpus == 1 and a.warmup >= 3 and a.impl == "ours"
    assert a.workload == "gauss-1m-d96" and a.batch == 10_000 and a.k == 10
    assert a.search_mode == "rabitq_gpu" and a.bits == 4 and a.mode == "search"
    wp = bench.workload_params(a.workload, a.n)
    assert (wp["n"], wp["dim"], wp["R"], wp["build_L"], wp["search_L"]) == (1_000_000, 96, 32, 128, 64)


def test_metric_name_names_the_mode():
    assert bench.metric_name(10, 64, "rabitq_gpu") == "queries/sec at recall@10 parity (k=10, L=64)"
    assert bench.metric_name(10, 64, "exact_gpu") == "queries/sec at recall@10 parity (k=10, L=64, exact_gpu)"


def test_bytes_per_query_formula():
    # 4D + H(4R+1) + E*S_code + C_r*4D + 4D^2/nq + 8k with S_code = ceil(B*D/8) + 8
    D, R, B, k, H, E, Cr, nq = 96, 32, 4, 10, 150.0, 4700.0, 128.0, 10_000
    s_code = (B * D + 7) // 8 + 8
    assert s_code == 56
    want = 4 * D + H * (4 * R + 1) + E * s_code + Cr * 4 * D + 4 * D * D / nq + 8 * k
    assert bench.bytes_per_query(D, R, B, k, H, E, Cr, nq) == pytest.approx(want)
    # exact_gpu: full vectors per distance, no rerank, no rotation
    assert bench.bytes_per_query(D, R, B, k, H, E, 0.0, nq, "exact_gpu") == pytest.approx(
        4 * D + H * (4 * R + 1) + E * 4 * D + 8 * k)


def test_profile_traffic_only_for_the_profiled_workload_and_sources():
    a = _args()
    wp = bench.workload_params(a.workload, a.n)
    tr, src = bench.profile_traffic(a, wp)
    digest = None
    for ln in open(bench.PROFILE_SUMMARY):
        if ln.startswith("kernel_sources_sha256_16="):
            digest = ln.split("=", 1)[1].split()[0]
    if digest == bench.kernel_sources_digest():
        assert tr is not None and tr > 1e9
    else:  # a capture of older kernel sources is not reported as this kernel's traffic
        assert tr is None and "does not match" in src
    for argv in (["--workload", "lowrank-1m-d960"], ["--search-mode", "exact_gpu"], ["--bits", "8"],
                 ["--k", "100"], ["--batch", "1000"], ["--n", "200000"]):
        b = _args(*argv)
        assert bench.profile_traffic(b, bench.workload_params(b.workload, b.n))[0] is None


def test_index_cache_tag_follows_the_bit_width():
    a4, a8 = _args(), _args("--bits", "8")
    wp = bench.workload_params(a4.workload)
    assert bench.index_prefix(a4, wp) != bench.index_prefix(a8, wp)
    assert "_b8_" in bench.index_prefix(a8, wp)


def test_launch_count_follows_the_prepare_kernels():
    # search kernel + prepare: tensor-core rotation and factors (2), FP32 rotation with
    # factors in one kernel up to 128 dims (1) or two above; exact_gpu has no prepare
    assert bench.launches_per_search(_args(), 96) == 3
    assert bench.launches_per_search(_args("--rotation", "exact"), 96) == 2
    assert bench.launches_per_search(_args("--rotation", "exact"), 960) == 3
    assert bench.launches_per_search(_args("--search-mode", "exact_gpu"), 96) == 1


def test_rotation_default_per_mode():
    # the search modes rotate on the tensor cores; the serving mix, whose small
    # query batches run beside insert kernels, on the FP32 pipe
    assert _args().rotation == "tensor"
    assert _args("--mode", "insert").rotation == "tensor"
    assert _args("--mode", "mixed").rotation == "exact"
    assert _args("--mode", "mixed", "--rotation", "tensor").rotation == "tensor"
    assert _args("--rotation", "exact").rotation == "exact"
