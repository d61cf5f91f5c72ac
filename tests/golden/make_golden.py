"""Records outputs of the reference's own GPU kernels as golden fixtures.

    python tests/golden/make_golden.py OUT_DIR

Needs a CUDA device and oracle/_ref/libref_gpu.so (the reference's
src/gpu/gpu_kernel_launcher.cu compiled from its sources by oracle/ref.mk).
Inputs are seeded; RaBitQ records, rotations and factors come from the
oracle.  Each .npz holds `kind`, the inputs and the reference output `out`
(or `q_rot`/`factor` for the query prepare).  The reference's L2 kernel reads
rows with uint4 loads, so only dims that are multiples of 4 are recorded.
"""
import ctypes as C
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import oracle as O  # noqa: E402


def main(out_dir):
    import torch

    os.makedirs(out_dir, exist_ok=True)
    lib = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref_gpu.so"))
    vp, u32 = C.c_void_p, C.c_uint32
    lib.ref_batch_rabitq_distances.argtypes = [vp, vp, vp, vp, u32, u32, u32]
    lib.ref_batch_l2_distances.argtypes = [vp, vp, vp, u32, u32]
    lib.ref_query_prepare.argtypes = [vp, vp, vp, vp, vp, u32, u32]
    lib.ref_quantize_single.argtypes = [vp, vp, vp, vp, u32, u32, C.c_double]

    keep = []  # device buffers stay alive until the reference kernels have run

    def dev(a):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        keep.append(t)
        torch.cuda.synchronize()
        return t

    def p(t):
        return C.c_void_p(t.data_ptr())

    rng = np.random.default_rng(2024)
    for bits, dim, n in [(4, 96, 512), (4, 128, 512), (4, 960, 128), (2, 96, 256), (1, 128, 256), (4, 40, 256)]:
        X = rng.standard_normal((n, dim)).astype(np.float32)
        X /= np.linalg.norm(X, axis=1, keepdims=True)
        P = O.rotation_matrix(dim, 1234)
        c_rot = O.rotate(P, O.centroid(X))
        rec = O.quantize_batch(X, P, c_rot, O.t_const(dim, bits, 1234), bits)
        q = rng.standard_normal(dim).astype(np.float32)
        q_rot, f = O.query_prepare(q, P, c_rot, bits)
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        d_rec, d_q, d_f = dev(rec.reshape(-1)), dev(q_rot), dev(f)
        assert lib.ref_batch_rabitq_distances(p(d_q), p(d_f), p(d_rec), p(out), n, dim, bits) == 0
        np.savez(os.path.join(out_dir, f"rabitq_b{bits}_d{dim}.npz"), kind="rabitq", bits=bits, dim=dim, q_rot=q_rot,
                 factor=f, records=rec, out=out.cpu().numpy())
    for dim, n in [(96, 300), (128, 300), (960, 64), (4, 100), (20, 100)]:
        q = rng.standard_normal(dim).astype(np.float32)
        cand = rng.standard_normal((n, dim)).astype(np.float32)
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        assert lib.ref_batch_l2_distances(p(dev(q)), p(dev(cand)), p(out), n, dim) == 0
        np.savez(os.path.join(out_dir, f"l2_d{dim}.npz"), kind="l2", query=q, cand=cand, out=out.cpu().numpy())
    for dim, bits in [(96, 4), (128, 4), (960, 4), (40, 2)]:
        P = O.rotation_matrix(dim, 77)
        c_rot = rng.standard_normal(dim).astype(np.float32)
        q = rng.standard_normal(dim).astype(np.float32)
        rq = torch.empty(dim, dtype=torch.float32, device="cuda")
        fac = torch.empty(3, dtype=torch.float32, device="cuda")
        assert lib.ref_query_prepare(p(dev(q)), p(dev(P)), p(dev(c_rot)), p(rq), p(fac), dim, bits) == 0
        np.savez(os.path.join(out_dir, f"prepare_d{dim}_b{bits}.npz"), kind="prepare", bits=bits, query=q, P=P,
                 c_rot=c_rot, q_rot=rq.cpu().numpy(), factor=fac.cpu().numpy())
    for dim, bits in [(96, 4), (128, 4)]:
        X = rng.standard_normal((64, dim)).astype(np.float32)
        X /= np.linalg.norm(X, axis=1, keepdims=True)
        P = O.rotation_matrix(dim, 1234)
        c_rot = O.rotate(P, O.centroid(X))
        tc = O.t_const(dim, bits, 1234)
        rs = O.rabitq_size(dim, bits)
        outs = []
        for x in X:
            o = torch.zeros(rs, dtype=torch.uint8, device="cuda")
            assert lib.ref_quantize_single(p(dev(x)), p(dev(P)), p(dev(c_rot)), p(o), dim, bits, tc) == 0
            outs.append(o.cpu().numpy())
        np.savez(os.path.join(out_dir, f"quantize_d{dim}_b{bits}.npz"), kind="quantize", bits=bits, x=X, P=P,
                 c_rot=c_rot, t_const=tc, out=np.stack(outs))
    # 8-bit codes: batch_rabitq_8bit_distance_kernel reads records with char4
    # loads, so dims are multiples of 4 (a record stride of dim + 8 bytes then
    # keeps every load aligned).  Own seed: the fixtures above stay unchanged.
    rng8 = np.random.default_rng(2025)
    for dim, n in [(96, 512), (128, 256), (960, 128), (40, 256)]:
        X = rng8.standard_normal((n, dim)).astype(np.float32)
        X /= np.linalg.norm(X, axis=1, keepdims=True)
        P = O.rotation_matrix(dim, 1234)
        c_rot = O.rotate(P, O.centroid(X))
        rec = O.quantize_batch(X, P, c_rot, O.t_const(dim, 8, 1234), 8)
        q = rng8.standard_normal(dim).astype(np.float32)
        q_rot, f = O.query_prepare(q, P, c_rot, 8)
        out = torch.empty(n, dtype=torch.float32, device="cuda")
        d_rec, d_q, d_f = dev(rec.reshape(-1)), dev(q_rot), dev(f)
        assert lib.ref_batch_rabitq_distances(p(d_q), p(d_f), p(d_rec), p(out), n, dim, 8) == 0
        np.savez(os.path.join(out_dir, f"rabitq_b8_d{dim}.npz"), kind="rabitq", bits=8, dim=dim, q_rot=q_rot,
                 factor=f, records=rec, out=out.cpu().numpy())
    for dim in (96,):
        P = O.rotation_matrix(dim, 78)
        c_rot = rng8.standard_normal(dim).astype(np.float32)
        q = rng8.standard_normal(dim).astype(np.float32)
        rq = torch.empty(dim, dtype=torch.float32, device="cuda")
        fac = torch.empty(3, dtype=torch.float32, device="cuda")
        assert lib.ref_query_prepare(p(dev(q)), p(dev(P)), p(dev(c_rot)), p(rq), p(fac), dim, 8) == 0
        np.savez(os.path.join(out_dir, f"prepare_d{dim}_b8.npz"), kind="prepare", bits=8, query=q, P=P,
                 c_rot=c_rot, q_rot=rq.cpu().numpy(), factor=fac.cpu().numpy())
    for dim in (96,):
        X = rng8.standard_normal((64, dim)).astype(np.float32)
        X /= np.linalg.norm(X, axis=1, keepdims=True)
        P = O.rotation_matrix(dim, 1234)
        c_rot = O.rotate(P, O.centroid(X))
        tc = O.t_const(dim, 8, 1234)
        rs = O.rabitq_size(dim, 8)
        outs = []
        for x in X:
            o = torch.zeros(rs, dtype=torch.uint8, device="cuda")
            assert lib.ref_quantize_single(p(dev(x)), p(dev(P)), p(dev(c_rot)), p(o), dim, 8, tc) == 0
            outs.append(o.cpu().numpy())
        np.savez(os.path.join(out_dir, f"quantize_d{dim}_b8.npz"), kind="quantize", bits=8, x=X, P=P,
                 c_rot=c_rot, t_const=tc, out=np.stack(outs))
    print("golden fixtures written to", out_dir)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
