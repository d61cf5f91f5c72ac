"""Seeded synthetic workloads (numpy PCG64 streams).  No public dataset is used:
each generator draws vectors with the shapes and value distributions of the
named workload."""
from __future__ import annotations

import numpy as np


def uniform_int(n: int, dim: int, seed: int) -> np.ndarray:
    """Coordinates i.i.d. uniform integers 0..255 cast to float32."""
    return np.random.default_rng(seed).integers(0, 256, size=(n, dim)).astype(np.float32)


def normalized_gaussian(n: int, dim: int, seed, chunk: int = 1 << 18) -> np.ndarray:
    """i.i.d. N(0,1) rows, L2-normalised."""
    rng = np.random.default_rng(seed)
    out = np.empty((n, dim), np.float32)
    for s in range(0, n, chunk):
        x = rng.standard_normal((min(chunk, n - s), dim), dtype=np.float32)
        x /= np.linalg.norm(x, axis=1, keepdims=True)
        out[s:s + len(x)] = x
    return out


def gaussian_mixture(n: int, dim: int, seed, clusters: int = 1024, sigma: float = 20.0, chunk: int = 1 << 18):
    """Mixture of `clusters` Gaussians: centres uniform in [0,255]^dim, per-cluster
    sigma, clipped to [0,255] and rounded to integers.  The centres depend on
    the first entry of `seed` only, so queries drawn with a longer seed
    (`queries_for`) come from the same mixture as the data."""
    centre_seed = seed[0] if isinstance(seed, (list, tuple)) else seed
    centres = np.random.default_rng([centre_seed, 0xCE]).uniform(0, 255, size=(clusters, dim)).astype(np.float32)
    rng = np.random.default_rng(seed)
    out = np.empty((n, dim), np.float32)
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        c = rng.integers(0, clusters, size=m)
        x = centres[c] + sigma * rng.standard_normal((m, dim), dtype=np.float32)
        out[s:s + m] = np.rint(np.clip(x, 0, 255))
    return out


def low_rank_uniform(n: int, dim: int, seed, rank: int = 64, chunk: int = 1 << 16):
    """Uniform [0,1) plus a random rank-`rank` component, standardised per dim
    with the distribution's own mean (1/2) and variance (1/12 + the basis
    column's squared norm), so every draw of any size shares one scaling.
    The basis depends on the first entry of `seed` only; data and queries that
    share it (`queries_for`) come from the same distribution."""
    basis_seed = seed[0] if isinstance(seed, (list, tuple)) else seed
    basis = np.random.default_rng([basis_seed, 0xBA5E]).standard_normal((rank, dim)).astype(np.float32)
    basis /= np.float32(np.sqrt(rank))
    sd = np.sqrt(1.0 / 12.0 + (basis.astype(np.float64) ** 2).sum(0)).astype(np.float32)
    rng = np.random.default_rng(seed)
    out = np.empty((n, dim), np.float32)
    for s in range(0, n, chunk):
        m = min(chunk, n - s)
        x = rng.random((m, dim), dtype=np.float32) + rng.standard_normal((m, rank), dtype=np.float32) @ basis
        out[s:s + m] = (x - np.float32(0.5)) / sd
    return out


WORKLOADS = {
    # name: (generator, n, dim, data seed, R, build L, search L, k)
    "plumbing-10k-d128": (uniform_int, 10_000, 128, 0, 32, 128, 64, 10),
    "gauss-1m-d96": (normalized_gaussian, 1_000_000, 96, 2, 32, 128, 64, 10),
    "mixture-10m-d128": (gaussian_mixture, 10_000_000, 128, 3, 32, 128, 100, 10),
    "lowrank-1m-d960": (low_rank_uniform, 1_000_000, 960, 4, 48, 128, 200, 10),
    "gauss-2m-d768": (normalized_gaussian, 2_000_000, 768, 5, 32, 128, 64, 10),
}


def queries_for(name: str, nq: int, stream: int = 0) -> np.ndarray:
    """Queries drawn from the workload's distribution with an independent seed."""
    gen, _, dim, seed, *_ = WORKLOADS[name]
    if gen is uniform_int:
        return uniform_int(nq, dim, seed + 1 + 1000 * stream)
    return gen(nq, dim, [seed, 1, stream])
