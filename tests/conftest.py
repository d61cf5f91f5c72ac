import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); run with -m gpu")


def has_gpu() -> bool:
    try:
        import dvstor_b200

        return dvstor_b200.lib().dvs_device_count() > 0
    except Exception:
        return False


@pytest.fixture(scope="session")
def oracle():
    from oracle import oracle as O

    O.build()
    return O


@pytest.fixture(scope="session")
def dvs():
    import dvstor_b200
    from dvstor_b200.build import build

    build()
    return dvstor_b200


@pytest.fixture(scope="session")
def gpu(dvs):
    if dvs.lib().dvs_device_count() == 0:
        pytest.fail("no CUDA device visible to a test marked gpu")
    return dvs


def uniform_int_data(n, d, seed):
    """Coordinates i.i.d. uniform integers 0..255 cast to float (the plumbing workload)."""
    return np.random.default_rng(seed).integers(0, 256, size=(n, d)).astype(np.float32)


def normalized_gaussian(n, d, seed):
    x = np.random.default_rng(seed).standard_normal((n, d)).astype(np.float32)
    return x / np.linalg.norm(x, axis=1, keepdims=True)


def write_oracle_index(O, idx, path, num_memory_nodes=1):
    os.makedirs(os.path.dirname(path), exist_ok=True)
    O.write_shards(path, idx.X, idx.adj, idx.medoid, idx.records, idx.P, idx.c_rot, idx.t_const, idx.bits,
                   num_memory_nodes=num_memory_nodes, metric=idx.metric)
    return path


def assert_results_match(gpu_ids, gpu_d, orc_ids, orc_d, orc_beam_ids, orc_beam_d):
    """Distances equal bit for bit; ids equal except inside groups of exactly equal
    distance, where std::sort's order is unspecified (the one documented tie)."""
    assert gpu_d.dtype == np.float32 and orc_d.dtype == np.float32
    np.testing.assert_array_equal(gpu_d.view(np.uint32), orc_d.view(np.uint32))
    diff = np.argwhere(gpu_ids != orc_ids)
    for q, i in diff:
        d = gpu_d[q, i]
        group = set(orc_beam_ids[q][orc_beam_d[q] == d].tolist())
        assert int(gpu_ids[q, i]) in group, f"query {q} rank {i}: id {gpu_ids[q, i]} not in tie group {group}"
        assert (gpu_d[q] == d).sum() > 1 or (orc_beam_d[q] == d).sum() > 1, f"query {q} rank {i} differs without a tie"
    return len(diff)
