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
    # online insert: the GPU quantizer kernel and RobustPrune.  The quantizer is
    # driven through launch_rabitq_quantize_single with P = I, so cuBLAS's
    # rotation returns the input exactly and the fixture records the kernel's
    # own arithmetic on a known rotated vector.  That kernel stores its two
    # float factors at byte offset (bits*dim+7)/8 of the output, which is only
    # aligned when that offset is a multiple of 4: the other sizes make a
    # misaligned store, so only aligned sizes are recorded.
    lib.ref_robust_prune.argtypes = [vp, vp, vp, vp, u32, u32, C.c_float, u32, vp, vp]
    rngi = np.random.default_rng(2026)
    for bits, dim in [(4, 96), (4, 40), (8, 128), (2, 96), (1, 128)]:
        assert ((bits * dim + 7) // 8) % 4 == 0
        X = rngi.standard_normal((48, dim)).astype(np.float32)
        c_rot = (0.1 * rngi.standard_normal(dim)).astype(np.float32)
        eye = np.eye(dim, dtype=np.float32)
        tc = O.t_const(dim, bits, 1234)
        rs = O.rabitq_size(dim, bits)
        outs = []
        for x in X:
            o = torch.zeros(rs, dtype=torch.uint8, device="cuda")
            assert lib.ref_quantize_single(p(dev(x)), p(dev(eye)), p(dev(c_rot)), p(o), dim, bits, tc) == 0
            outs.append(o.cpu().numpy())
        np.savez(os.path.join(out_dir, f"quantize_gpu_d{dim}_b{bits}.npz"), kind="quantize_gpu", bits=bits,
                 x_rot=X, c_rot=c_rot, t_const=tc, out=np.stack(outs))
    for name, n, dim, R, alpha, permute in [("a", 120, 32, 16, 1.2, False), ("b", 120, 32, 16, 1.0, True),
                                            ("c", 10, 24, 16, 1.2, False), ("d", 65, 96, 64, 1.2, True)]:
        src = rngi.standard_normal(dim).astype(np.float32)
        V = (src + 0.5 * rngi.standard_normal((n, dim))).astype(np.float32)
        d = O.l2_batch(src, V)
        order = np.argsort(d, kind="stable").astype(np.uint32)
        if permute:
            cand, dists, ordv = V, d[order], order          # vectors in original order, order maps rank -> index
        else:
            cand, dists, ordv = V[order], d[order], None    # vectors already sorted
        out = torch.zeros(R, dtype=torch.int32, device="cuda")
        cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
        d_ord = dev(ordv) if ordv is not None else None
        assert lib.ref_robust_prune(p(dev(src)), p(dev(cand)), p(dev(dists)), p(d_ord) if d_ord is not None else None,
                                    n, dim, alpha, R, p(out), p(cnt)) == 0
        k = int(cnt.item())
        np.savez(os.path.join(out_dir, f"prune_{name}.npz"), kind="prune", cand=cand, dists=dists,
                 order=ordv if ordv is not None else np.zeros(0, np.uint32), alpha=np.float32(alpha), R=R,
                 out=out.cpu().numpy()[:k].astype(np.uint32))
    print("golden fixtures written to", out_dir)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.dirname(os.path.abspath(__file__)))
