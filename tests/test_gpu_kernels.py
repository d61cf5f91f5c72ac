"""GPU parity of the kernel-level entry points against the oracle, bit for bit:
dvs_l2_distances (gpu::launch_batch_l2_distances), dvs_rabitq_estimate
(gpu::launch_batch_rabitq_distances) and dvs_query_prepare
(gpu::launch_rabitq_query_prepare), called through the C ABI on device buffers."""
import ctypes as C

import numpy as np
import pytest

from conftest import normalized_gaussian

pytestmark = pytest.mark.gpu


def _dev(a):
    import torch

    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _sync():
    import torch

    torch.cuda.synchronize()


@pytest.mark.parametrize("dim", [1, 3, 4, 30, 96, 128, 131, 960])
def test_l2_distances_bit_exact(gpu, oracle, dim):
    import torch

    from dvstor_b200._lib import check, lib, ptr

    rng = np.random.default_rng(dim)
    q = rng.standard_normal(dim).astype(np.float32)
    x = rng.standard_normal((257, dim)).astype(np.float32)
    dq, dx = _dev(q), _dev(x)
    out = torch.empty(257, dtype=torch.float32, device="cuda")
    check(lib().dvs_l2_distances(ptr(dq), ptr(dx), ptr(out), 257, dim, None))
    _sync()
    ref = oracle.l2_batch(q, x)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("bits,dim", [(4, 96), (4, 128), (4, 33), (2, 96), (2, 70), (1, 128), (1, 100), (4, 960),
                                      (8, 96), (8, 960), (8, 30), (8, 130)])
def test_rabitq_estimate_bit_exact(gpu, oracle, bits, dim):
    import torch

    from dvstor_b200._lib import check, lib, ptr

    X = normalized_gaussian(300, dim, bits + dim)
    P = oracle.rotation_matrix(dim, 5)
    c_rot = oracle.rotate(P, oracle.centroid(X))
    rec = oracle.quantize_batch(X, P, c_rot, oracle.t_const(dim, bits, 5), bits)
    qr, f = oracle.query_prepare(normalized_gaussian(1, dim, 1)[0], P, c_rot, bits)
    d_rec, d_qr, d_f = _dev(rec.reshape(-1)), _dev(qr), _dev(f)
    out = torch.empty(300, dtype=torch.float32, device="cuda")
    check(lib().dvs_rabitq_estimate(ptr(d_qr), ptr(d_f), ptr(d_rec), ptr(out), 300, dim, bits, None))
    _sync()
    ref = oracle.rabitq_estimate(qr, f, rec, dim, bits)
    np.testing.assert_array_equal(out.cpu().numpy().view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("dim,bits,nq", [(96, 4, 37), (128, 4, 130), (30, 2, 37), (960, 4, 37), (960, 4, 130),
                                         (131, 4, 65), (200, 1, 64), (257, 4, 3)])
def test_query_prepare_bit_exact(gpu, oracle, dim, bits, nq):
    """Two kernels: P^T resident in shared memory (dim <= 128) and the
    register-tiled product (dim > 128); tile edges in both query and output."""
    import torch

    from dvstor_b200._lib import check, lib, ptr

    P = oracle.rotation_matrix(dim, 11)
    c_rot = np.random.default_rng(3).standard_normal(dim).astype(np.float32)
    Q = normalized_gaussian(nq, dim, 2)
    dQ, dP, dc = _dev(Q), _dev(P), _dev(c_rot)
    qr = torch.empty((nq, dim), dtype=torch.float32, device="cuda")
    fac = torch.empty((nq, 3), dtype=torch.float32, device="cuda")
    check(lib().dvs_query_prepare(ptr(dQ), ptr(dP), ptr(dc), ptr(qr), ptr(fac), nq, dim, bits, None))
    _sync()
    for i in range(nq):
        rq, rf = oracle.query_prepare(Q[i], P, c_rot, bits)
        np.testing.assert_array_equal(qr[i].cpu().numpy().view(np.uint32), rq.view(np.uint32))
        np.testing.assert_array_equal(fac[i].cpu().numpy().view(np.uint32), rf.view(np.uint32))


def test_kernel_entry_points_reject_bad_arguments(gpu):
    from dvstor_b200._lib import lib

    L = lib()
    one = C.c_void_p(1)
    assert L.dvs_rabitq_estimate(one, one, one, one, 4, 8, 3, None) == 5  # DVS_ERR_BITS
    assert L.dvs_l2_distances(one, one, one, 4, 0, None) == 4             # DVS_ERR_DIM
    assert L.dvs_l2_distances(one, one, one, 0, 8, None) == 0             # empty batch: no launch


@pytest.mark.parametrize("dim,nq", [(96, 300), (128, 129), (30, 5), (200, 64), (960, 130)])
def test_query_prepare_tensor_cores_accuracy(gpu, oracle, dim, nq):
    """tcgen05 3xTF32 rotation: within 1e-5 of the row's largest |q'| of the fp64
    product (fp32-level accuracy); factors equal the reference arithmetic applied
    to its rotated rows, bit for bit."""
    import torch

    from dvstor_b200._lib import check, lib, ptr

    P = oracle.rotation_matrix(dim, 13)
    c_rot = np.random.default_rng(4).standard_normal(dim).astype(np.float32)
    Q = np.random.default_rng(dim).standard_normal((nq, dim)).astype(np.float32)
    dQ, dP, dc = _dev(Q), _dev(P), _dev(c_rot)
    qr = torch.empty((nq, dim), dtype=torch.float32, device="cuda")
    fac = torch.empty((nq, 3), dtype=torch.float32, device="cuda")
    check(lib().dvs_query_prepare_tc(ptr(dQ), ptr(dP), ptr(dc), ptr(qr), ptr(fac), nq, dim, 4, None))
    _sync()
    got = qr.cpu().numpy()
    ref = Q.astype(np.float64) @ P.reshape(dim, dim).astype(np.float64).T  # row j of P.reshape = column j of P
    scale = np.abs(ref).max(axis=1, keepdims=True)
    assert (np.abs(got - ref) / scale).max() < 1e-5
    f = fac.cpu().numpy()
    for i in range(0, nq, max(1, nq // 7)):
        np.testing.assert_array_equal(f[i].view(np.uint32), oracle.query_factors(got[i], c_rot, 4).view(np.uint32))
