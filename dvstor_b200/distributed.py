"""One process per GPU: replicas of the index, a query batch split across ranks.

Queries are independent, so multi-GPU serving needs no collective on the data
path: every rank holds a replica (or, within one process, a shard set opened
with placement="shard").  `chunk_bounds` is the split rule dvs_search uses
across the devices of one process (contiguous chunks, q0 = nq*i/n);
`ReplicaSearch` applies it across torchrun ranks: rank 0 holds the batch,
scatters the chunks, every rank searches its own chunk on its own GPU and the
results are gathered back to rank 0.  The process group may be NCCL (tensors
on the rank's GPU) or gloo (host tensors).
"""
from __future__ import annotations

import numpy as np


def chunk_bounds(n: int, world: int, rank: int) -> tuple[int, int]:
    """[begin, end) of rank's contiguous share of n items."""
    return n * rank // world, n * (rank + 1) // world


class ReplicaSearch:
    """Scatter / search / gather over a torch.distributed process group.

    `search_fn(queries: np.ndarray (m, dim)) -> (ids (m, k) uint32, dists (m, k) float32)`
    runs on every rank (normally `Index.search` of the rank's own replica)."""

    def __init__(self, search_fn, dim: int, k: int, group=None, device=None):
        import torch.distributed as dist

        self.dist = dist
        self.search_fn = search_fn
        self.dim = dim
        self.k = k
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = device  # torch device of the rank's tensors (cuda for NCCL, cpu for gloo)

    def _t(self, a):
        import torch

        t = torch.from_numpy(np.ascontiguousarray(a))
        return t.to(self.device) if self.device is not None else t

    def search(self, queries=None):
        """Rank 0 passes the (nq, dim) batch, the others None; rank 0 gets (ids, dists)."""
        import torch

        dist, world, rank = self.dist, self.world, self.rank
        n = torch.zeros(1, dtype=torch.int64)
        if rank == 0:
            n[0] = queries.shape[0]
        n = self._t(n.numpy())
        dist.broadcast(n, 0, group=self.group)
        nq = int(n.item())
        per = max((nq + world - 1) // world, 1)
        # rank 0 pads the batch to world * per rows so every chunk has one shape
        buf = np.zeros((world * per, self.dim), np.float32)
        if rank == 0:
            for r in range(world):
                b0, b1 = chunk_bounds(nq, world, r)
                buf[r * per:r * per + (b1 - b0)] = queries[b0:b1]
        full = self._t(buf)
        dist.broadcast(full, 0, group=self.group)
        b0, b1 = chunk_bounds(nq, world, rank)
        mine = full[rank * per:rank * per + (b1 - b0)].cpu().numpy()
        ids, dists = self.search_fn(mine) if b1 > b0 else (np.zeros((0, self.k), np.uint32),
                                                            np.zeros((0, self.k), np.float32))
        out_i = np.zeros((per, self.k), np.int64)
        out_d = np.zeros((per, self.k), np.float32)
        out_i[:b1 - b0] = ids.astype(np.int64)
        out_d[:b1 - b0] = dists
        gi = [self._t(np.zeros_like(out_i)) for _ in range(world)]
        gd = [self._t(np.zeros_like(out_d)) for _ in range(world)]
        dist.all_gather(gi, self._t(out_i), group=self.group)
        dist.all_gather(gd, self._t(out_d), group=self.group)
        if rank != 0:
            return None
        res_i = np.empty((nq, self.k), np.uint32)
        res_d = np.empty((nq, self.k), np.float32)
        for r in range(world):
            c0, c1 = chunk_bounds(nq, world, r)
            res_i[c0:c1] = gi[r].cpu().numpy()[:c1 - c0].astype(np.uint32)
            res_d[c0:c1] = gd[r].cpu().numpy()[:c1 - c0]
        return res_i, res_d
