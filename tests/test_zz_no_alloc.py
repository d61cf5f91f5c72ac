"""dvs_search_device_noalloc: the device-resident search for callers that may
not allocate device memory once running (for example a serving engine that
has reserved the GPU's free memory for its own pool, so any later cudaMalloc
fails).  It must return exactly what dvs_search_device returns, on two calls
in a row (its fixed scratch keeps the previous call's contents, spill tables
included), without changing the device's free memory, and reject batches
beyond its fixed scratch with a clear error.

This file is collected last so that a run stopping at the first failure has
already run every other test."""
import ctypes as C

import numpy as np
import pytest

from conftest import normalized_gaussian, write_oracle_index

pytestmark = pytest.mark.gpu

MAX_QUERY_BYTES = (8 << 20) - 256  # the rotated-query region of the fixed scratch


def _noalloc(ix, dq, k, L, mode, out_ids, out_d, cnt, stream):
    from dvstor_b200._lib import check, lib, ptr

    check(lib().dvs_search_device_noalloc(ix._h, 0, ptr(dq), dq.shape[0], dq.shape[1], k, L,
                                          0 if mode == "rabitq_gpu" else 1, ptr(out_ids), ptr(out_d), ptr(cnt),
                                          C.c_void_p(stream.cuda_stream)))


def _compare_two_calls(ix, Q, k, L, mode):
    """dvs_search_device once, then the no-allocation search twice in a row;
    ids, distances and per-query counters equal, free device memory unchanged
    on the second call (the first may load the module that holds the array)."""
    import torch

    nq = Q.shape[0]
    stream = torch.cuda.Stream()
    dq = torch.from_numpy(Q).cuda()
    ref_ids = torch.empty((nq, k), dtype=torch.int32, device="cuda")
    ref_d = torch.empty((nq, k), dtype=torch.float32, device="cuda")
    ref_c = torch.zeros((nq, 4), dtype=torch.int32, device="cuda")
    ix.search_device(dq, k, L, mode, d_out_ids=ref_ids, d_out_dist=ref_d, d_counters=ref_c, stream=stream)
    torch.cuda.synchronize()
    outs = []
    for call in range(2):
        ids = torch.full((nq, k), -7, dtype=torch.int32, device="cuda")
        d = torch.full((nq, k), -7.0, dtype=torch.float32, device="cuda")
        c = torch.zeros((nq, 4), dtype=torch.int32, device="cuda")
        torch.cuda.synchronize()
        free0 = torch.cuda.mem_get_info()[0]
        _noalloc(ix, dq, k, L, mode, ids, d, c, stream)
        torch.cuda.synchronize()
        if call == 1:
            assert torch.cuda.mem_get_info()[0] == free0
        outs.append((ids.cpu().numpy(), d.cpu().numpy(), c.cpu().numpy()))
    for ids, d, c in outs:
        np.testing.assert_array_equal(ids, ref_ids.cpu().numpy())
        np.testing.assert_allclose(d, ref_d.cpu().numpy(), rtol=0, atol=0)
        np.testing.assert_array_equal(c, ref_c.cpu().numpy())
    return ref_c.cpu().numpy()


@pytest.fixture(scope="module")
def small_index(oracle, tmp_path_factory):
    X = normalized_gaussian(4000, 64, 31)
    idx = oracle.build_index(X, R=24, L=48)
    return idx, write_oracle_index(oracle, idx, str(tmp_path_factory.mktemp("noalloc") / "idx"))


@pytest.mark.parametrize("mode,L", [("rabitq_gpu", 64), ("exact_gpu", 48)])
def test_noalloc_matches_device_search(gpu, small_index, mode, L):
    _, pre = small_index
    with gpu.Index(pre) as ix:
        _compare_two_calls(ix, normalized_gaussian(700, 64, 32), 10, L, mode)


@pytest.mark.parametrize("mode,L", [("rabitq_gpu", 64), ("exact_gpu", 64)])
def test_noalloc_spill_tables_back_to_back(gpu, small_index, mode, L):
    """Two slots per beam entry: every query outgrows the shared-memory table
    and continues in its warp's spill table, which the second call finds
    holding the first call's entries."""
    _, pre = small_index
    Q = normalized_gaussian(700, 64, 34)
    with gpu.Index(pre) as ix:
        ix.set_visited_slots(2)
        _, _, st = ix.search(Q, 10, L, mode, stats=True)
        assert st["overflow_queries"] > 0
        cnt = _compare_two_calls(ix, Q, 10, L, mode)
        assert not (cnt[:, 3] >> 16).any()  # no query ran out of capacity


def test_noalloc_tensor_rotation(gpu, small_index):
    """With the rotation on tensor cores both entry points rotate the same way."""
    _, pre = small_index
    with gpu.Index(pre) as ix:
        ix.set_rotation("tensor")
        _compare_two_calls(ix, normalized_gaussian(300, 64, 35), 10, 64, "rabitq_gpu")


def test_noalloc_largest_batch(gpu, oracle, tmp_path):
    """The largest batch the fixed scratch takes at dim 96."""
    X = normalized_gaussian(3000, 96, 36)
    idx = oracle.build_index(X, R=16, L=32)
    pre = write_oracle_index(oracle, idx, str(tmp_path / "idx"))
    nq = MAX_QUERY_BYTES // (96 * 4 + 16)
    with gpu.Index(pre) as ix:
        _compare_two_calls(ix, normalized_gaussian(nq, 96, 37), 10, 32, "rabitq_gpu")


def test_noalloc_empty_index(gpu, small_index):
    import torch

    idx, _ = small_index
    ix = gpu.Index.create(64, 24, idx.P, idx.c_rot, idx.t_const, rabitq_bits=4)
    try:
        dq = torch.from_numpy(normalized_gaussian(5, 64, 38)).cuda()
        ids = torch.zeros((5, 10), dtype=torch.int32, device="cuda")
        d = torch.zeros((5, 10), dtype=torch.float32, device="cuda")
        c = torch.full((5, 4), 7, dtype=torch.int32, device="cuda")
        stream = torch.cuda.Stream()
        _noalloc(ix, dq, 10, 32, "rabitq_gpu", ids, d, c, stream)
        stream.synchronize()
        assert (ids.cpu().numpy().view(np.uint32) == 0xFFFFFFFF).all()
        assert np.isinf(d.cpu().numpy()).all()
        assert (c.cpu().numpy() == 0).all()
    finally:
        ix.close()


def test_noalloc_rejects_batches_beyond_its_scratch(gpu, oracle, tmp_path):
    import torch

    X = normalized_gaussian(600, 96, 33)
    idx = oracle.build_index(X, R=16, L=32)
    pre = write_oracle_index(oracle, idx, str(tmp_path / "idx"))
    nq = MAX_QUERY_BYTES // (96 * 4 + 16) + 1
    with gpu.Index(pre) as ix:
        dq = torch.zeros((nq, 96), dtype=torch.float32, device="cuda")
        ids = torch.empty((nq, 10), dtype=torch.int32, device="cuda")
        d = torch.empty((nq, 10), dtype=torch.float32, device="cuda")
        with pytest.raises(gpu.DvsError) as e:
            _noalloc(ix, dq, 10, 32, "rabitq_gpu", ids, d, None, torch.cuda.Stream())
        assert e.value.name == "DVS_ERR_CAPACITY" and "at most" in str(e.value)
