#!/usr/bin/env python
"""Throughput of the rabitq_gpu query path: queries/sec at fixed beam width and k.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (default): 1,000,000 x 96 fp32 vectors, i.i.d. N(0,1) then
L2-normalised (seed 2); Vamana R=32, build L=128, RaBitQ 4-bit; search k=10,
beam L=64.  One step = one batch of 10,000 queries (same distribution) searched
by one persistent kernel per GPU; with N GPUs every rank holds a replica of the
index and searches its own 10,000-query batch per step (weak scaling, no
collective on the data path).  The index (0.58 GB of adjacency, records and
vectors) is larger than L2, which is not flushed between steps.

`value`   device-resident queries -> device results (CUDA events, max over ranks).
`e2e`     the public host API (dvs_search): pinned host queries in, host ids and
          distances out, copies inside the timed region (wall clock per rank, max
          over ranks).
`--impl reference` times the reference's CPU Vamana beam search (restated in
oracle/, the reference's own code cannot be built here) on the host cores.

The query rotation runs on the tcgen05 tensor cores (`--rotation tensor`, the
default of the search modes; the parity leg then gives the oracle the GPU's
rotated queries) or on the FP32 pipe in the oracle's own order (`--rotation
exact`, the default of `--mode mixed`: its query batches hold a few queries and
run beside insert kernels, where the tensor-core kernel's large shared-memory
stage waits for a free SM).

Other rows of the path: `--search-mode exact_gpu` (exact L2 for every
candidate), `--bits 1|2|8` (the index built with that code width),
`--workload` / `--n` / `--batch` / `--k` / `--beam-width` for the other
workloads, `--placement shard` (one process, the index split over --gpus
devices), `--mode insert|mixed` (online insert, and queries interleaved with
inserts).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOAD = "gauss-1m-d96"
BATCH = 10_000
PEAKS = os.path.join(ROOT, "MEASURED_PEAKS.json")
PROFILE_SUMMARY = os.path.join(ROOT, "profiles", "search_kernel_gauss-1m-d96.txt")


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=WORKLOAD)
    ap.add_argument("--beam-width", type=int, default=None)
    ap.add_argument("--k", type=int, default=10)
    ap.add_argument("--search-mode", choices=["rabitq_gpu", "exact_gpu"], default="rabitq_gpu",
                    help="exact_gpu: exact L2 for every candidate, no estimate and no rerank")
    ap.add_argument("--bits", type=int, choices=[1, 2, 4, 8], default=4, help="RaBitQ code width of the index")
    ap.add_argument("--batch", type=int, default=BATCH)
    ap.add_argument("--n", type=int, default=None, help="index size override (reduced-size runs of a workload)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="target CPU time of the cpu_baseline sample")
    ap.add_argument("--cache", default=os.environ.get("DVS_BENCH_CACHE", "/tmp/dvs_b200_bench"))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--mode", choices=["search", "insert", "mixed"], default="search",
                    help="insert: online insert throughput (dvs_insert); mixed: queries and inserts interleaved")
    ap.add_argument("--insert-count", type=int, default=100_000)
    ap.add_argument("--insert-batch", type=int, default=4096)
    ap.add_argument("--beam-width-construction", type=int, default=128)
    ap.add_argument("--alpha", type=float, default=1.2)
    ap.add_argument("--placement", choices=["replicate", "shard"], default="replicate",
                    help="shard: one process over --gpus devices, the index split by slot (run without torchrun)")
    ap.add_argument("--rotation", choices=["exact", "tensor"], default=None,
                    help="query rotation: tcgen05 tensor cores (3xTF32; the default except in --mode mixed), or fp32 "
                         "in the oracle's fixed order (the default of --mode mixed)")
    ap.add_argument("--metric", choices=["l2", "ip"], default=None,
                    help="index metric (default: ip for --mode mixed, else l2)")
    ap.add_argument("--clients", type=int, default=16, help="--mode mixed: client threads per GPU")
    ap.add_argument("--read-ratio", type=float, default=0.5, help="--mode mixed: fraction of operations that are queries")
    ap.add_argument("--seconds", type=float, default=20.0, help="--mode mixed: measured seconds")
    ap.add_argument("--warmup-seconds", type=float, default=5.0, help="--mode mixed: warm-up seconds")
    ap.add_argument("--reserve", type=int, default=400_000, help="--mode mixed: insert capacity reserved up front")
    ap.add_argument("--report", default=None, help="--mode mixed: path of the breakdown JSON report")
    ap.add_argument("--parity-queries", type=int, default=500,
                    help="queries of the workload checked against the oracle's Vamana::knn after the timed region")
    ap.add_argument("--build-index-only", action="store_true", help=argparse.SUPPRESS)
    args = ap.parse_args()
    if args.rotation is None:
        args.rotation = "exact" if args.mode == "mixed" else "tensor"
    return args


def log(*a):
    print(*a, file=sys.stderr, flush=True)


_RESULT_FD = None


def emit(line: dict) -> None:
    """The one JSON result line, on the process's original stdout."""
    fd = _RESULT_FD if _RESULT_FD is not None else sys.stdout.fileno()
    os.write(fd, (json.dumps(line) + "\n").encode())


def route_stdout_to_stderr() -> None:
    """Libraries print to file descriptor 1 (NCCL announces its version there when
    a communicator comes up); send all of it to stderr so stdout carries only the
    result line."""
    global _RESULT_FD
    sys.stdout.flush()
    _RESULT_FD = os.dup(1)
    os.dup2(2, 1)


class Dist:
    """torch.distributed plumbing when launched by torchrun."""

    def __init__(self, backend):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist

            dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, x: float) -> float:
        if not self.pg:
            return x
        import torch

        dev = f"cuda:{self.local}" if self.pg.get_backend() == "nccl" else "cpu"
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


def workload_params(name, n=None):
    from dvstor_b200 import datasets

    gen, n0, dim, seed, R, build_L, search_L, k = datasets.WORKLOADS[name]
    return dict(gen=gen, n=n or n0, dim=dim, seed=seed, R=R, build_L=build_L, search_L=search_L, k=k)


def index_metric(args) -> str:
    return args.metric or ("ip" if args.mode == "mixed" else "l2")


def index_prefix(args, wp):
    tag = f"{args.workload}_n{wp['n']}_R{wp['R']}_L{wp['build_L']}_b{args.bits}_s1234"
    if index_metric(args) != "l2":
        tag += f"_{index_metric(args)}"
    return os.path.join(args.cache, tag, "idx")


def ensure_index(args, wp, device, dist, subprocess_build=False):
    """Builds the index once per box (GPU builder) into the cache directory.
    subprocess_build: build in a child process, so this process never loads
    the library (the reference arm)."""
    prefix = index_prefix(args, wp)
    done = prefix + ".done"
    if dist.local == 0 and not os.path.exists(done) and subprocess_build:
        cmd = [sys.executable, os.path.abspath(__file__), "--build-index-only", "--workload", args.workload,
               "--bits", str(args.bits), "--cache", args.cache, "--metric", index_metric(args)]
        if args.n:
            cmd += ["--n", str(args.n)]
        subprocess.run(cmd, check=True, stdout=sys.stderr)
    if dist.local == 0 and not os.path.exists(done):
        from dvstor_b200.builder import build_index

        t = time.time()
        X = wp["gen"](wp["n"], wp["dim"], wp["seed"])
        log(f"[bench] generated {X.shape} in {time.time() - t:.1f}s; building index on cuda:{device}")
        t = time.time()
        st = build_index(X, prefix, R=wp["R"], beam_width=wp["build_L"], alpha=1.2, rabitq_bits=args.bits,
                         seed=1234, device=device, metric=index_metric(args))
        log(f"[bench] built in {time.time() - t:.1f}s ({st})")
        open(done, "w").write(json.dumps(st))
    dist.barrier()
    return prefix


def clocks_sampler(device):
    """nvidia-smi clock/throttle sampling during the timed region."""
    q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")
    try:
        p = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-i", str(device),
                              "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
    except OSError:
        return None
    lines = []

    def reader():
        for ln in p.stdout:
            lines.append((time.time(), ln))

    th = threading.Thread(target=reader, daemon=True)
    th.start()
    time.sleep(0.5)  # nvidia-smi needs a moment before its first sample
    return p, lines, th


def clocks_summary(sampler, t0=None, t1=None):
    """Median SM clock and throttle reasons of the samples taken in [t0, t1]."""
    if sampler is None:
        return None
    p, stamped, th = sampler
    p.terminate()
    try:
        p.wait(timeout=5)
    except subprocess.TimeoutExpired:
        p.kill()
    th.join(timeout=2)
    sm, mx, reasons = [], [], set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    inside = [ln for ts, ln in stamped if t0 is None or t0 - 0.06 <= ts <= t1 + 0.06]
    for ln in inside:
        f = [x.strip() for x in ln.split(",")]
        if len(f) < 9:
            continue
        try:
            sm.append(float(f[1]))
            mx.append(float(f[2]))
        except ValueError:
            continue
        for nm, v in zip(names, f[5:9]):
            if v.lower() == "active":
                reasons.add(nm)
    if not sm:
        return None
    return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons), "samples": len(sm)}


def ground_truth(X, Q, k, device):
    """Exact top-k by brute force on the GPU (fp32, TF32 off), chunked over queries."""
    import torch

    torch.backends.cuda.matmul.allow_tf32 = False
    dev = torch.device(f"cuda:{device}")
    Xt = torch.from_numpy(X).to(dev)
    xx = (Xt.double() ** 2).sum(1).float()
    out = []
    for s in range(0, len(Q), 256):
        q = torch.from_numpy(Q[s:s + 256]).to(dev)
        d = xx[None, :] - 2.0 * (q @ Xt.T)
        out.append(torch.topk(d, k, dim=1, largest=False).indices.cpu().numpy())
    del Xt
    torch.cuda.empty_cache()
    return np.concatenate(out)


def recall(ids, gt):
    k = gt.shape[1]
    return float(np.mean([len(set(ids[i][:k].tolist()) & set(gt[i].tolist())) / k for i in range(len(gt))]))


def tensor_rotated(ix, Q, device):
    """The rotated queries and factors the tensor-core rotation gives for this
    index (dvs_query_prepare_tc with the index's P and rotated centroid)."""
    import torch

    from dvstor_b200._lib import check, lib, ptr

    P, c = ix.artifacts()
    dev = f"cuda:{device}"
    dQ, dP, dc = (torch.from_numpy(np.ascontiguousarray(a)).to(dev) for a in (Q, P, c))
    qr = torch.empty(Q.shape, dtype=torch.float32, device=dev)
    fac = torch.empty((Q.shape[0], 3), dtype=torch.float32, device=dev)
    check(lib().dvs_query_prepare_tc(ptr(dQ), ptr(dP), ptr(dc), ptr(qr), ptr(fac), Q.shape[0], Q.shape[1],
                                     ix.info.rabitq_bits, None))
    torch.cuda.synchronize(device)
    return qr.cpu().numpy(), fac.cpu().numpy()


def parity_check(ix, orc, Q, k, L, mode, device, rotation="exact"):
    """The GPU search against the oracle's Vamana::knn (src/vamana/vamana.hh:57-452)
    on the same index files and queries: a query matches when its distances are
    equal bit for bit, its expansions H, estimates E and reranked rows C_r are
    equal, and its ids are equal except inside groups of exactly equal final
    distance (std::sort leaves their order unspecified).  With the tensor-core
    rotation the oracle is given the GPU's rotated queries and factors."""
    import torch

    nq = Q.shape[0]
    dev = f"cuda:{device}"
    dq = torch.from_numpy(np.ascontiguousarray(Q)).to(dev)
    ids_t = torch.empty((nq, k), dtype=torch.int32, device=dev)
    d_t = torch.empty((nq, k), dtype=torch.float32, device=dev)
    c_t = torch.zeros((nq, 4), dtype=torch.int32, device=dev)
    ix.search_device(dq, k, L, mode, d_out_ids=ids_t, d_out_dist=d_t, d_counters=c_t)
    torch.cuda.synchronize(device)
    g_ids = ids_t.cpu().numpy().view(np.uint32)
    g_d = d_t.cpu().numpy()
    g_c = c_t.cpu().numpy().view(np.uint32)
    cap = L + 64 if mode == "rabitq_gpu" else L
    t = time.perf_counter()
    q_rot = fac = None
    if rotation == "tensor" and mode == "rabitq_gpu":
        q_rot, fac = tensor_rotated(ix, Q, device)
    o_ids, o_d, o_c, b_ids, b_d = orc.knn(Q, k, L, mode, q_rot=q_rot, factors=fac, beam_cap=cap,
                                          threads=os.cpu_count() or 1)
    oracle_s = time.perf_counter() - t
    mism, ties = 0, 0
    for q in range(nq):
        ok = np.array_equal(g_d[q].view(np.uint32), o_d[q].view(np.uint32)) and np.array_equal(g_c[q, :3], o_c[q, :3])
        if ok:
            for i in np.nonzero(g_ids[q] != o_ids[q])[0]:
                dv = g_d[q, i]
                tie = (g_d[q] == dv).sum() > 1 or (b_d[q] == dv).sum() > 1
                if tie and int(g_ids[q, i]) in set(b_ids[q][b_d[q] == dv].tolist()):
                    ties += 1
                else:
                    ok = False
        mism += 0 if ok else 1
    rule = "distances and H/E/C_r equal bit for bit, ids equal outside exact-distance ties"
    if q_rot is not None:
        rule += "; the oracle given the GPU's tensor-core rotated queries"
    return {"queries": nq, "mismatches": mism, "tie_diffs": ties, "oracle_s": round(oracle_s, 2), "rule": rule}


def index_device_bytes(info):
    """HBM bytes of one replica: adjacency, records (16-byte padded), vectors, ids."""
    rec = (((info.rabitq_bits * info.dim + 7) // 8 + 3) // 4 * 4 + 8 + 15) // 16 * 16
    vec = (info.dim + 3) // 4 * 16
    return info.num_vectors * (4 * info.R + rec + vec + 4)


def bytes_per_query(dim, R, bits, k, H, E, Cr, nq, mode="rabitq_gpu"):
    """Algorithmic bytes of one query: query row, H adjacency rows (R ids + count),
    E RaBitQ records (codes + add + rescale), C_r rerank rows, the rotation
    matrix amortised over the batch, and k (id, distance) results.  exact_gpu
    reads E full vectors instead of records and has no rerank or rotation."""
    if mode == "exact_gpu":
        return 4 * dim + H * (4 * R + 1) + E * 4 * dim + 8 * k
    s_code = (bits * dim + 7) // 8 + 8
    return 4 * dim + H * (4 * R + 1) + E * s_code + Cr * 4 * dim + 4 * dim * dim / nq + 8 * k


def launches_per_search(args, dim) -> int:
    """This library's kernels per search call: the search kernel, and for
    rabitq_gpu the query prepare (the tensor-core rotation and the factors
    kernel; the FP32 rotation with its factors in one kernel up to 128 dims,
    in two above)."""
    if args.search_mode == "exact_gpu":
        return 1
    if args.rotation == "tensor" or dim > 128:
        return 3
    return 2


def metric_name(k, L, mode):
    """The headline metric; exact_gpu runs name their mode."""
    return f"queries/sec at recall@10 parity (k={k}, L={L}{', exact_gpu' if mode == 'exact_gpu' else ''})"


MODE_ID = {"rabitq_gpu": 0, "exact_gpu": 1}  # dvs_mode


KERNEL_SOURCES = ("search.cu", "search.cuh", "device_math.cuh", "api.cu", "index_state.h")


def kernel_sources_digest() -> str:
    """sha256 (first 16 hex digits) of the sources that decide what the search
    kernel reads and writes: the kernel, its launch shape and its scratch."""
    import hashlib

    h = hashlib.sha256()
    for f in KERNEL_SOURCES:
        h.update(open(os.path.join(ROOT, "dvstor_b200", "csrc", f), "rb").read())
    return h.hexdigest()[:16]


def profile_traffic(args, wp):
    """DRAM bytes per launch of the search kernel from the committed ncu summary:
    (bytes, provenance).  The summary covers the default workload only and names
    the digest of the kernel sources it was captured from; for any other
    configuration, or when the sources have changed since, bytes is None."""
    if (args.workload, wp["n"], args.batch, args.k, args.beam_width, args.search_mode, args.bits) != (
            WORKLOAD, workload_params(WORKLOAD)["n"], BATCH, 10, None, "rabitq_gpu", 4):
        return None, "no ncu capture of this configuration"
    tr, digest = None, None
    try:
        for ln in open(PROFILE_SUMMARY):
            if ln.startswith("traffic_bytes_per_launch_full_workload="):
                tr = float(ln.split("=", 1)[1].split()[0])
            if ln.startswith("kernel_sources_sha256_16="):
                digest = ln.split("=", 1)[1].split()[0]
    except OSError:
        return None, "no ncu summary"
    src = f"ncu capture in profiles/{os.path.basename(PROFILE_SUMMARY)} (kernel sources {digest})"
    if tr is None or digest != kernel_sources_digest():
        return None, src + f" does not match the current kernel sources ({kernel_sources_digest()})"
    return tr, src


def hbm_peak():
    try:
        return float(json.load(open(PEAKS))["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def cpu_baseline(idx_or, Q, L, k, target_s, gt_q=None):
    """The reference's CPU beam search over a bounded query sample, all host threads."""
    from oracle import oracle as O

    cores = os.cpu_count() or 1
    probe = Q[:min(len(Q), 2000)]
    t = time.perf_counter()
    O.cpu_beam_search_batch(idx_or.X, idx_or.adj, idx_or.medoid, probe, L, k, threads=cores)
    qps0 = len(probe) / (time.perf_counter() - t)
    n = int(min(len(Q), max(len(probe), qps0 * target_s)))
    sample = Q[:n]
    t = time.perf_counter()
    ids, _ = O.cpu_beam_search_batch(idx_or.X, idx_or.adj, idx_or.medoid, sample, L, k, threads=cores)
    el = time.perf_counter() - t
    rec = recall(ids, gt_q) if gt_q is not None else None
    return {"value": n / el, "unit": "queries/s", "cores": cores, "kind": "port",
            "sample": f"{n} queries of the workload, beam_search (exact L2, L={L}) per query, "
                      f"{cores} threads, {el:.1f}s", "recall_at_10": rec}


def run_reference(args):
    dist = Dist("gloo")
    if dist.rank != 0:
        dist.close()
        return
    from dvstor_b200 import datasets
    from oracle import oracle as O

    wp = workload_params(args.workload, args.n)
    L = args.beam_width or wp["search_L"]
    dist_single = Dist.__new__(Dist)
    dist_single.world, dist_single.rank, dist_single.local, dist_single.pg = 1, 0, 0, None
    prefix = ensure_index(args, wp, 0, dist_single, subprocess_build=True)
    idx = O.read_index(prefix)
    cores = os.cpu_count() or 1
    Qpool = datasets.queries_for(args.workload, 200_000, stream=0)
    t = time.perf_counter()
    O.cpu_beam_search_batch(idx.X, idx.adj, idx.medoid, Qpool[:1000], L, args.k, threads=cores)
    qps0 = 1000 / (time.perf_counter() - t)
    per_step = int(min(len(Qpool), max(1000, qps0 * 8.0)))  # ~8 s of CPU work per step
    for s in range(args.warmup):
        O.cpu_beam_search_batch(idx.X, idx.adj, idx.medoid, Qpool[:min(per_step, 2000)], L, args.k, threads=cores)
    times = []
    for s in range(args.steps):
        q = np.roll(Qpool, -s * 997, axis=0)[:per_step]
        t = time.perf_counter()
        O.cpu_beam_search_batch(idx.X, idx.adj, idx.medoid, q, L, args.k, threads=cores)
        times.append(time.perf_counter() - t)
    qps = per_step * len(times) / sum(times)
    gt = ground_truth(idx.X, Qpool[:1000], args.k, 0)
    ids, _ = O.cpu_beam_search_batch(idx.X, idx.adj, idx.medoid, Qpool[:1000], L, args.k, threads=cores)
    line = {
        "impl": "reference", "metric": metric_name(args.k, L, args.search_mode), "value": qps,
        "unit": "queries/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * sum(times) / len(times), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "n": wp["n"], "dim": wp["dim"], "R": wp["R"], "build_L": wp["build_L"],
                   "rabitq_bits": args.bits, "search_mode": args.search_mode, "k": args.k, "beam_width": L,
                   "queries_per_step": per_step, "l2": "index larger than L2, not flushed"},
        "cpu_baseline": {"value": qps, "unit": "queries/s", "cores": cores, "kind": "port",
                         "sample": f"{per_step} queries per step, the reference's CPU beam_search restated "
                                   f"(tools/vamana_offline_builder.cc:523-625), {cores} threads"},
        "e2e": {"value": qps, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "recall_at_10": recall(ids, gt),
    }
    emit(line)


def run_ours(args):
    import torch

    dist = Dist("nccl")
    device = dist.local
    torch.cuda.set_device(device)
    import dvstor_b200 as D
    from dvstor_b200 import datasets

    wp = workload_params(args.workload, args.n)
    L = args.beam_width or wp["search_L"]
    k = args.k
    B = args.batch
    prefix = ensure_index(args, wp, device, dist)
    ix = D.Index(prefix, devices=(device,))
    ix.set_rotation(args.rotation)
    info = ix.info
    nsteps = args.warmup + args.steps
    Qpool = datasets.queries_for(args.workload, B * nsteps, stream=dist.rank)
    dq = torch.from_numpy(Qpool).to(f"cuda:{device}").view(nsteps, B, wp["dim"])
    out_ids = torch.empty((B, k), dtype=torch.int32, device=f"cuda:{device}")
    out_d = torch.empty((B, k), dtype=torch.float32, device=f"cuda:{device}")
    cnt = torch.zeros((B, 4), dtype=torch.int32, device=f"cuda:{device}")
    stream = torch.cuda.Stream(device=device)

    # ---- device-resident timed region ----
    with torch.cuda.stream(stream):
        for s in range(args.warmup):
            ix.search_device(dq[s], k, L, args.search_mode, d_out_ids=out_ids, d_out_dist=out_d, d_counters=cnt,
                             stream=stream)
    torch.cuda.synchronize(device)
    ix.set_kernel_timing(True)
    ix.kernel_times()
    sampler = clocks_sampler(device)
    dist.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_wall0 = time.time()
    e0.record(stream)
    for s in range(args.steps):
        ix.search_device(dq[args.warmup + s], k, L, args.search_mode, d_out_ids=out_ids, d_out_dist=out_d,
                         d_counters=cnt, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize(device)
    t_wall1 = time.time()
    dist.barrier()
    clocks = clocks_summary(sampler, t_wall0, t_wall1)
    ms = e0.elapsed_time(e1)
    n_search, prep_ms, search_ms = ix.kernel_times()
    ix.set_kernel_timing(False)
    ms_max = dist.max(ms)
    value = dist.world * B * args.steps / (ms_max / 1e3)

    # per-query work of the last step -> algorithmic bytes
    c = cnt.cpu().numpy().astype(np.int64)
    H, E, Cr = c[:, 0].mean(), c[:, 1].mean(), c[:, 2].mean()
    bq = bytes_per_query(info.dim, info.R, info.rabitq_bits, k, H, E, Cr, B, args.search_mode)
    search_avg_ms = search_ms / max(n_search, 1)
    achieved = bq * B / (search_avg_ms / 1e3) / 1e9
    peak, peak_kind = hbm_peak()
    tr, tr_src = profile_traffic(args, wp)
    prep_avg_ms = prep_ms / max(n_search, 1)

    # ---- end to end through the host API ----
    # every step's queries are staged in pinned host memory before timing; a
    # step is one dvs_search call: H2D of the batch, prepare + search, D2H of
    # ids and distances into pinned buffers
    hq_all = torch.empty((nsteps, B, wp["dim"]), dtype=torch.float32, pin_memory=True).numpy()
    hq_all[:] = Qpool.reshape(nsteps, B, wp["dim"])
    h_ids = torch.empty((B, k), dtype=torch.int32, pin_memory=True).numpy().view(np.uint32)
    h_d = torch.empty((B, k), dtype=torch.float32, pin_memory=True).numpy()
    from dvstor_b200._lib import check, lib, ptr

    def host_search(s):
        check(lib().dvs_search(ix._h, ptr(hq_all[s]), B, wp["dim"], k, L, MODE_ID[args.search_mode], ptr(h_ids),
                               ptr(h_d), None))

    for s in range(min(args.warmup, 2)):
        host_search(s)
    dist.barrier()
    e2e_times = []
    for s in range(args.steps):
        step_i = (args.warmup + s) % nsteps
        t = time.perf_counter()
        host_search(step_i)
        e2e_times.append(time.perf_counter() - t)
    e2e_s = dist.max(sum(e2e_times))
    e2e = dist.world * B * args.steps / e2e_s

    # ---- recall and the CPU baseline (rank 0) ----
    rec = cpu = par = None
    if dist.rank == 0:
        from oracle import oracle as O

        X = O.read_index(prefix)
        Xv = X.X
        gtq = Qpool[:1000]
        g_ids, _ = ix.search(gtq, k, L, args.search_mode)
        gt = ground_truth(Xv, gtq, k, device)
        rec = recall(g_ids, gt)
        if args.parity_queries:
            par = parity_check(ix, X, Qpool[:args.parity_queries], k, L, args.search_mode, device, args.rotation)
        if not args.no_cpu_baseline and dist.world == 1:  # timed at N=1 only
            cpu = cpu_baseline(X, np.concatenate([gtq, Qpool[1000:]]), L, k, args.cpu_seconds, gt_q=None)
            ids_cpu, _ = O.cpu_beam_search_batch(X.X, X.adj, X.medoid, gtq, L, k)
            cpu["recall_at_10"] = recall(ids_cpu, gt)
    ix.close()
    if dist.rank == 0:
        line = {
            "metric": metric_name(k, L, args.search_mode), "value": value, "unit": "queries/s",
            "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": args.workload, "n": wp["n"], "dim": wp["dim"], "R": wp["R"],
                       "build_L": wp["build_L"], "rabitq_bits": args.bits, "search_mode": args.search_mode, "k": k,
                       "beam_width": L, "rotation": args.rotation, "queries_per_step_per_gpu": B,
                       "parallelism": f"replicas x{dist.world}",
                       "l2": f"index {index_device_bytes(info) / 1e9:.2f} GB larger than L2, not flushed; "
                             "fresh query batch every step"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": tr, "traffic_source": tr_src,
                         "peak_source": f"{peak_kind} hbm_gbs", "kernel": "search_kernel",
                         "kernel_ms": search_avg_ms, "prepare_ms": prep_avg_ms,
                         "bytes_per_query": bq,
                         "per_query": {"H": H, "E": E, "C_r": Cr, "E_p99": float(np.percentile(c[:, 1], 99)),
                                       "E_max": int(c[:, 1].max())}},
            "e2e": {"value": e2e, "unit": "queries/s", "h2d_bytes_per_step": B * wp["dim"] * 4,
                    "d2h_bytes_per_step": B * k * 8},
            "gpu_launches": launches_per_search(args, wp["dim"]) * args.steps,
            "clocks": clocks,
            "recall_at_10": rec,
            "parity": par,
            "cpu_baseline": cpu,
        }
        emit(line)
    dist.barrier()
    dist.close()


def run_sharded(args):
    """One process over --gpus devices with the index split by slot (placement
    "shard": node g on device g mod N, remote rows read from peer HBM).  Every
    device searches its own batch per step on its own stream; time = max over
    devices of the CUDA-event time."""
    import torch

    import dvstor_b200 as D
    from dvstor_b200 import datasets

    ngpu = args.gpus
    dist = Dist("gloo")
    wp = workload_params(args.workload, args.n)
    L = args.beam_width or wp["search_L"]
    k, B = args.k, args.batch
    prefix = ensure_index(args, wp, 0, dist)
    ix = D.Index(prefix, devices=tuple(range(ngpu)), placement="shard")
    ix.set_rotation(args.rotation)
    info = ix.info
    nsteps = args.warmup + args.steps
    Qpool = datasets.queries_for(args.workload, B * ngpu * nsteps)
    per = Qpool.reshape(nsteps, ngpu, B, wp["dim"])
    dq = [torch.from_numpy(np.ascontiguousarray(per[:, d])).to(f"cuda:{d}") for d in range(ngpu)]
    outs = [(torch.empty((B, k), dtype=torch.int32, device=f"cuda:{d}"),
             torch.empty((B, k), dtype=torch.float32, device=f"cuda:{d}"),
             torch.zeros((B, 4), dtype=torch.int32, device=f"cuda:{d}")) for d in range(ngpu)]
    streams = [torch.cuda.Stream(device=d) for d in range(ngpu)]

    def step(s):
        for d in range(ngpu):
            with torch.cuda.device(d):
                ix.search_device(dq[d][s], k, L, args.search_mode, d_out_ids=outs[d][0], d_out_dist=outs[d][1],
                                 d_counters=outs[d][2], stream=streams[d], device_slot=d)

    for s in range(args.warmup):
        step(s)
    for d in range(ngpu):
        torch.cuda.synchronize(d)
    ix.set_kernel_timing(True)
    for d in range(ngpu):
        ix.kernel_times(d)
    sampler = clocks_sampler(0)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(ngpu)]
    t_wall0 = time.time()
    for d in range(ngpu):
        ev[d][0].record(streams[d])
    for s in range(args.steps):
        step(args.warmup + s)
    for d in range(ngpu):
        ev[d][1].record(streams[d])
    for d in range(ngpu):
        torch.cuda.synchronize(d)
    t_wall1 = time.time()
    clocks = clocks_summary(sampler, t_wall0, t_wall1)
    ms = max(ev[d][0].elapsed_time(ev[d][1]) for d in range(ngpu))
    ktimes = [ix.kernel_times(d) for d in range(ngpu)]
    ix.set_kernel_timing(False)
    value = ngpu * B * args.steps / (ms / 1e3)
    c = np.concatenate([outs[d][2].cpu().numpy() for d in range(ngpu)]).astype(np.int64)
    H, E, Cr = c[:, 0].mean(), c[:, 1].mean(), c[:, 2].mean()
    bq = bytes_per_query(info.dim, info.R, info.rabitq_bits, k, H, E, Cr, B, args.search_mode)
    search_avg_ms = max(st / max(n, 1) for n, _, st in ktimes)
    achieved = bq * B * ngpu / (search_avg_ms / 1e3) / 1e9
    peak, peak_kind = hbm_peak()

    # end to end: dvs_search splits a host batch over the devices
    hq = torch.empty((B * ngpu, wp["dim"]), dtype=torch.float32, pin_memory=True)
    h_ids = torch.empty((B * ngpu, k), dtype=torch.int32, pin_memory=True).numpy().view(np.uint32)
    h_d = torch.empty((B * ngpu, k), dtype=torch.float32, pin_memory=True).numpy()
    from dvstor_b200._lib import check, lib, ptr

    def host_search(q):
        hq.numpy()[:] = q
        check(lib().dvs_search(ix._h, ptr(hq.numpy()), B * ngpu, wp["dim"], k, L, MODE_ID[args.search_mode],
                               ptr(h_ids), ptr(h_d), None))

    host_search(per[0].reshape(-1, wp["dim"]))
    t = time.perf_counter()
    for s in range(args.steps):
        host_search(per[(args.warmup + s) % nsteps].reshape(-1, wp["dim"]))
    e2e = ngpu * B * args.steps / (time.perf_counter() - t)

    gtq = Qpool[:1000]
    g_ids, _ = ix.search(gtq, k, L, args.search_mode)
    Xv = ix.download()[2]
    rec = recall(g_ids, ground_truth(Xv, gtq, k, 0))
    ix.close()
    line = {
        "metric": metric_name(k, L, args.search_mode), "value": value, "unit": "queries/s",
        "n_gpus": ngpu, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "n": wp["n"], "dim": wp["dim"], "R": wp["R"], "build_L": wp["build_L"],
                   "rabitq_bits": args.bits, "search_mode": args.search_mode, "k": k, "beam_width": L,
                   "rotation": args.rotation, "queries_per_step_per_gpu": B,
                   "parallelism": f"shard x{ngpu} (one process, peer HBM reads)",
                   "l2": f"index {index_device_bytes(info) / 1e9:.2f} GB split over {ngpu} GPUs, not flushed"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak * ngpu, "unit": "GB/s",
                     "frac": achieved / (peak * ngpu), "traffic": None,
                     "peak_source": f"{peak_kind} hbm_gbs x {ngpu} GPUs", "kernel": "search_kernel",
                     "kernel_ms": search_avg_ms, "bytes_per_query": bq, "per_query": {"H": H, "E": E, "C_r": Cr}},
        "e2e": {"value": e2e, "unit": "queries/s", "h2d_bytes_per_step": B * ngpu * wp["dim"] * 4,
                "d2h_bytes_per_step": B * ngpu * k * 8},
        "gpu_launches": launches_per_search(args, wp["dim"]) * args.steps * ngpu,
        "clocks": clocks,
        "recall_at_10": rec,
        "cpu_baseline": None,
    }
    emit(line)


def run_insert(args):
    """Online insert throughput (Vamana::insert, src/vamana/vamana.hh:458-999):
    --insert-count new vectors of the workload's distribution go into the base
    index through dvs_insert (host vectors in, steps of at most --insert-batch),
    wall clock around each call; the oracle's CPU insert on a bounded sample of
    the same stream is the baseline."""
    import torch

    import dvstor_b200 as D
    from dvstor_b200 import datasets

    dist = Dist("gloo")
    wp = workload_params(args.workload, args.n)
    prefix = ensure_index(args, wp, 0, dist)
    torch.cuda.set_device(0)
    ix = D.Index(prefix, devices=(0,))
    n0 = int(ix.info.num_vectors)
    B, Lc, total = args.insert_batch, args.beam_width_construction, args.insert_count
    warm = args.warmup * B
    Xn = datasets.queries_for(args.workload, warm + total, stream=9)
    ids = np.arange(n0, n0 + warm + total, dtype=np.uint32)
    ix.reserve(n0 + warm + total)
    ix.insert(Xn[:warm], ids[:warm], beam_width_construction=Lc, alpha=args.alpha, max_batch=B)
    torch.cuda.synchronize()
    sampler = clocks_sampler(0)
    t_wall0 = time.time()
    stats = {"expansions": 0, "distances": 0, "full_prunes": 0, "steps": 0, "device_ms": 0.0, "prune_ms": 0.0,
             "reverse_ms": 0.0, "max_incoming": 0}
    t = time.perf_counter()
    for s in range(warm, warm + total, B):
        st = ix.insert(Xn[s:s + B], ids[s:s + B], beam_width_construction=Lc, alpha=args.alpha, max_batch=B)
        for key in stats:
            stats[key] = max(stats[key], st[key]) if key == "max_incoming" else stats[key] + st[key]
    el = time.perf_counter() - t
    clocks = clocks_summary(sampler, t_wall0, time.time())
    value = total / el
    # the inserted vectors are found again (rank 0 = themselves)
    probe = slice(warm, warm + min(total, 2000))
    got, _ = ix.search(Xn[probe], 10, 64)
    self_hit = float((got[:, 0] == ids[probe]).mean())
    ix.close()
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import oracle as O

        orc = O.read_index(prefix)
        cores = os.cpu_count() or 1
        m = min(total, max(B, 2000))
        t = time.perf_counter()
        orc.insert(Xn[warm:warm + m], ids[warm:warm + m], beam_width_construction=Lc, alpha=args.alpha, max_batch=B,
                   threads=cores)
        cel = time.perf_counter() - t
        cpu = {"value": m / cel, "unit": "inserts/s", "cores": cores, "kind": "port",
               "sample": f"{m} inserts into the same base index, Vamana::insert restated (steps of {B}, searches "
                         f"on {cores} threads, reverse edges sequential), {cel:.1f}s"}
    line = {
        "metric": f"inserts/sec (L_c={Lc}, alpha={args.alpha})", "value": value, "unit": "inserts/s",
        "n_gpus": 1, "steps": stats["steps"], "warmup": args.warmup, "ms_per_step": 1e3 * el / max(stats["steps"], 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.workload, "n_base": n0, "dim": wp["dim"], "R": wp["R"], "rabitq_bits": args.bits,
                   "inserted": total, "insert_batch": B, "beam_width_construction": Lc, "alpha": args.alpha},
        "e2e": {"value": value, "unit": "inserts/s", "h2d_bytes_per_step": B * wp["dim"] * 4 + B * 4,
                "d2h_bytes_per_step": B * wp["R"] * 4},
        "insert_stats": stats, "self_hit_at_1": self_hit, "gpu_launches": 7 * stats["steps"],
        "clocks": clocks, "cpu_baseline": cpu,
    }
    emit(line)


def run_mixed(args):
    """The dynamic serving mix (Vamana::knn and Vamana::insert served
    concurrently): --clients client threads per GPU, each issuing one operation
    at a time and waiting for it, a query (k, beam width) with probability
    --read-ratio and otherwise a single-vector insert (beam width
    construction, alpha), for --seconds after --warmup-seconds; the
    inner-product metric by default.  Operations go through
    dvstor_b200.serving.BatchingServer (pending queries batched into one
    dvs_search call, pending inserts into one dvs_insert call).  Reports
    operations/s, queries/s, inserts/s and p50/p95/p99 latency per operation,
    and writes the reference's breakdown JSON report (--report).  Under
    torchrun every rank serves its own replica with its own clients and
    inserts (weak scaling); time = max over ranks."""
    import torch

    import dvstor_b200 as D
    from dvstor_b200 import datasets
    from dvstor_b200.serving import BatchingServer, Breakdown

    dist = Dist("nccl" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "gloo")
    device = dist.local
    torch.cuda.set_device(device)
    wp = workload_params(args.workload, args.n)
    L = args.beam_width or wp["search_L"]
    k = args.k
    prefix = ensure_index(args, wp, device, dist)
    ix = D.Index(prefix, devices=(device,))
    ix.set_rotation(args.rotation)
    n0 = int(ix.info.num_vectors)
    ix.reserve(n0 + args.reserve)
    bd = Breakdown()
    server = BatchingServer(ix, k, L, args.search_mode, args.beam_width_construction, args.alpha, breakdown=bd)
    Qpool = datasets.queries_for(args.workload, 65536, stream=3 + 100 * dist.rank)
    Xpool = datasets.queries_for(args.workload, 65536, stream=9 + 100 * dist.rank)
    id_lock = threading.Lock()
    next_id = [n0]
    inserted = []
    phase = {"measure": False, "stop": False}
    counts = {"query": 0, "insert": 0}

    def client(c):
        rng = np.random.default_rng([5, dist.rank, c])
        i = c
        while not phase["stop"]:
            if rng.random() < args.read_ratio:
                server.search(Qpool[i % len(Qpool)])
                kind = "query"
            else:
                with id_lock:
                    ident = next_id[0]
                    next_id[0] += 1
                server.insert(ident, Xpool[(ident - n0) % len(Xpool)])
                inserted.append(ident)
                kind = "insert"
            if phase["measure"]:
                counts[kind] += 1
            i += args.clients

    threads = [threading.Thread(target=client, args=(c,), daemon=True) for c in range(args.clients)]
    dist.barrier()
    for t in threads:
        t.start()
    time.sleep(args.warmup_seconds)
    bd.__init__()  # the report covers the measured window only
    batches0 = dict(server.batches)
    sampler = clocks_sampler(device)
    t_wall0 = time.time()
    t0 = time.perf_counter()
    phase["measure"] = True
    time.sleep(args.seconds)
    phase["measure"] = False
    el = time.perf_counter() - t0
    t_wall1 = time.time()
    phase["stop"] = True
    for t in threads:
        t.join()
    server.close()
    clocks = clocks_summary(sampler, t_wall0, t_wall1)
    batches = {kk: server.batches[kk] - batches0[kk] for kk in batches0}
    rep = bd.report(meta={"client_threads": args.clients, "read_ratio": args.read_ratio, "dim": wp["dim"],
                          "search_mode": args.search_mode, "measure_seconds": args.seconds,
                          "warmup_seconds": args.warmup_seconds, "operation_granularity": "single_vector",
                          "workload": "mixed", "batching": "pending queries per dvs_search, pending inserts "
                                                           "per dvs_insert", "rank": dist.rank})
    # the inserted vectors are found again (rank 0 = themselves)
    probe = np.array(inserted[:1000], np.int64)
    self_hit = None
    if len(probe):
        got, _ = ix.search(Xpool[(probe - n0) % len(Xpool)], 10, L, args.search_mode)
        self_hit = float((got[:, 0] == probe.astype(np.uint32)).mean())
    ix.close()
    el_max = dist.max(el)
    tot_q = counts["query"]
    if dist.world > 1:
        import torch.distributed as tdist

        t = torch.tensor([counts["query"], counts["insert"]], dtype=torch.float64, device=f"cuda:{device}")
        tdist.all_reduce(t)
        tot_q, tot_i = float(t[0]), float(t[1])
    else:
        tot_i = counts["insert"]
    if args.report:
        path = args.report if dist.world == 1 else f"{args.report}.rank{dist.rank}"
        os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
        open(path, "w").write(json.dumps(rep, indent=2, sort_keys=True))

    def lat(op):
        j = rep.get(f"{op}_breakdown")
        if not j:
            return None
        l_ = j["latency"]
        return {"count": j["count"], "mean_ms": l_["mean_end_to_end_ns"] / 1e6, "p50_ms": l_["p50_end_to_end_ns"] / 1e6,
                "p95_ms": l_["p95_end_to_end_ns"] / 1e6, "p99_ms": l_["p99_end_to_end_ns"] / 1e6,
                "mean_queue_wait_ms": l_["mean_queue_wait_ns"] / 1e6, "gpu_share": (
                    j["breakdown"]["gpu_ns"] / l_["service_ns"] if l_["service_ns"] else None)}

    if dist.rank == 0:
        ops = (tot_q + tot_i) / el_max
        line = {
            "metric": f"operations/sec, {args.clients} client streams per GPU, {int(args.read_ratio * 100)}% queries "
                      f"(k={k}, L={L}) / single-vector inserts (L_c={args.beam_width_construction})",
            "value": ops, "unit": "ops/s", "n_gpus": dist.world, "steps": args.seconds, "warmup": args.warmup_seconds,
            "ms_per_step": None, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": args.workload, "n_base": n0, "dim": wp["dim"], "R": wp["R"],
                       "rabitq_bits": args.bits, "metric": args.metric or "ip", "clients_per_gpu": args.clients,
                       "read_ratio": args.read_ratio, "measure_seconds": args.seconds,
                       "parallelism": f"replicas x{dist.world}, each with its own clients and inserts"},
            "queries_per_s": tot_q / el_max, "inserts_per_s": tot_i / el_max,
            "latency": {"query": lat("query"), "insert": lat("insert")},
            "batches": batches, "self_hit_at_1": self_hit,
            "e2e": {"value": ops, "unit": "ops/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": None},
            "clocks": clocks, "report": args.report,
        }
        emit(line)
    dist.barrier()
    dist.close()


def main():
    args = parse_args()
    route_stdout_to_stderr()
    if args.build_index_only:
        single = Dist.__new__(Dist)
        single.world, single.rank, single.local, single.pg = 1, 0, 0, None
        ensure_index(args, workload_params(args.workload, args.n), 0, single)
        return
    if args.impl == "reference":
        run_reference(args)
    elif args.mode == "insert":
        run_insert(args)
    elif args.mode == "mixed":
        run_mixed(args)
    elif args.placement == "shard":
        run_sharded(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
