"""dvs_search_device_noalloc: the device-resident search for callers that may
not allocate device memory once running (for example a serving engine that
has reserved the GPU's free memory for its own pool).  It must return exactly
what dvs_search_device returns, on two calls in a row (its fixed scratch keeps
the previous call's contents), without changing the device's free memory, and
reject batches beyond its fixed scratch with a clear error.

This file is collected last so that a run stopping at the first failure has
already run every other test."""
import os

import numpy as np
import pytest

from conftest import normalized_gaussian, write_oracle_index

pytestmark = pytest.mark.gpu


def _noalloc(ix, dq, k, L, mode, out_ids, out_d, cnt, stream):
    from dvstor_b200._lib import check, lib, ptr

    import ctypes as C

    check(lib().dvs_search_device_noalloc(ix._h, 0, ptr(dq), dq.shape[0], dq.shape[1], k, L,
                                          0 if mode == "rabitq_gpu" else 1, ptr(out_ids), ptr(out_d), ptr(cnt),
                                          C.c_void_p(stream.cuda_stream)))


@pytest.mark.parametrize("mode,L", [("rabitq_gpu", 64), ("exact_gpu", 48)])
def test_noalloc_matches_device_search(gpu, oracle, tmp_path, mode, L):
    import torch

    X = normalized_gaussian(4000, 64, 31)
    Q = normalized_gaussian(700, 64, 32)
    idx = oracle.build_index(X, R=24, L=48)
    pre = write_oracle_index(oracle, idx, str(tmp_path / "idx"))
    with gpu.Index(pre) as ix:
        stream = torch.cuda.Stream()
        dq = torch.from_numpy(Q).cuda()
        ref_ids = torch.empty((700, 10), dtype=torch.int32, device="cuda")
        ref_d = torch.empty((700, 10), dtype=torch.float32, device="cuda")
        ref_c = torch.zeros((700, 4), dtype=torch.int32, device="cuda")
        ix.search_device(dq, 10, L, mode, d_out_ids=ref_ids, d_out_dist=ref_d, d_counters=ref_c, stream=stream)
        outs = []
        for call in range(2):
            ids = torch.full((700, 10), -7, dtype=torch.int32, device="cuda")
            d = torch.full((700, 10), -7.0, dtype=torch.float32, device="cuda")
            c = torch.zeros((700, 4), dtype=torch.int32, device="cuda")
            torch.cuda.synchronize()
            free0 = torch.cuda.mem_get_info()[0]
            _noalloc(ix, dq, 10, L, mode, ids, d, c, stream)
            torch.cuda.synchronize()
            if call == 1:  # the first call may load the module that holds the fixed array
                assert torch.cuda.mem_get_info()[0] == free0
            outs.append((ids.cpu().numpy(), d.cpu().numpy(), c.cpu().numpy()))
        torch.cuda.synchronize()
        for ids, d, c in outs:
            np.testing.assert_array_equal(ids, ref_ids.cpu().numpy())
            np.testing.assert_allclose(d, ref_d.cpu().numpy(), rtol=0, atol=0)
            np.testing.assert_array_equal(c, ref_c.cpu().numpy())


def test_noalloc_rejects_batches_beyond_its_scratch(gpu, oracle, tmp_path):
    import torch

    X = normalized_gaussian(600, 96, 33)
    idx = oracle.build_index(X, R=16, L=32)
    pre = write_oracle_index(oracle, idx, str(tmp_path / "idx"))
    nq = (8 << 20) // (96 * 4 + 16) + 1
    with gpu.Index(pre) as ix:
        dq = torch.zeros((nq, 96), dtype=torch.float32, device="cuda")
        ids = torch.empty((nq, 10), dtype=torch.int32, device="cuda")
        d = torch.empty((nq, 10), dtype=torch.float32, device="cuda")
        with pytest.raises(gpu.DvsError) as e:
            _noalloc(ix, dq, 10, 32, "rabitq_gpu", ids, d, None, torch.cuda.Stream())
        assert e.value.name == "DVS_ERR_CAPACITY" and "at most" in str(e.value)
