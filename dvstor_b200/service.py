"""Flag-compatible front end of the reference's compute-node service.

The reference configures ComputeService from command-line flags
(boost::program_options, src/common/configuration.hh:87-154) and checks them in
validate_compute_node_options (:156-198).  ``parse_config`` accepts the same
flags, aliases and defaults, applies the checks that concern a compute node
with an HBM-resident index, and raises ``ConfigError`` with the reference's
messages instead of exiting.  ``Service`` is ComputeService over this
library: ``search`` / ``insert`` / ``load_index`` / ``store_index`` /
``status`` (src/service/compute_service.hh:84-103) plus the per-operation
counters of statistics::ThreadStatistics (src/common/statistics.hh:188-251)
that the GPU path produces.

Flags that configure the RDMA transport, CPU caches, coroutine and worker
counts are accepted (so existing command lines still parse) and recorded, but
have nothing to configure here: the index lives in HBM and one kernel answers
a batch.
"""
from __future__ import annotations

import argparse
import dataclasses
import os

import numpy as np

SEARCH_MODES = ("exact_gpu", "rabitq_gpu")
RABITQ_BITS = (1, 2, 4, 8)


class ConfigError(ValueError):
    """A flag combination the reference rejects (it prints the message and exits)."""


@dataclasses.dataclass
class ServiceConfig:
    data_path: str = ""
    index_prefix: str = ""
    threads: int = 0
    coroutines: int = 4
    disable_thread_pinning: bool = False
    seed: int = 1234
    label: str = ""
    query_suffix: str = ""
    store_index: bool = False
    load_index: bool = False
    cache: bool = False
    routing: bool = False
    cache_ratio: int = 5
    no_recall: bool = False
    ip_dist: bool = False
    beam_width: int = 0
    beam_width_construction: int = 200
    k: int = 0
    R: int = 64
    alpha: float = 1.2
    rabitq_bits: int = 1
    search_mode: str = "exact_gpu"
    insert_workers: int = 0
    query_workers: int = 0
    insert_coroutines: int = 0
    query_coroutines: int = 0
    gpu_device: int = 0
    gpudirect_rdma: bool = False
    neighbor_cache_mb: int = 0
    gpu_rabitq_cache_mb: int = 0
    dim: int = 0
    max_vectors: int = 1_000_000
    cn_memory: int = 10
    mn_memory: int = 10

    def resolved_index_prefix(self) -> str:
        """index_path::resolve_prefix (src/common/index_path.hh:14-24): the explicit
        prefix, else <data dir>/dump/index_m<R>_efc<beam_width_construction>."""
        if self.index_prefix:
            return self.index_prefix
        if not self.data_path:
            raise ConfigError("data path must not be empty")
        base = os.path.dirname(self.data_path) if os.path.splitext(self.data_path)[1] else self.data_path
        return os.path.join(base, "dump", f"index_m{self.R}_efc{self.beam_width_construction}")


def build_parser() -> argparse.ArgumentParser:
    """The flags of IndexConfiguration::add_options (configuration.hh:87-154)."""
    ap = argparse.ArgumentParser(prog="dvstor-compute", allow_abbrev=False)
    a = ap.add_argument
    a("--data-path", "-d", dest="data_path", default="")
    a("--index-prefix", dest="index_prefix", default="")
    a("--server-index-file", dest="server_index_file", default="")
    a("--threads", "-t", dest="threads", type=int, default=0)
    a("--coroutines", "-C", dest="coroutines", type=int, default=4)
    a("--disable-thread-pinning", "-p", dest="disable_thread_pinning", action="store_true")
    a("--seed", dest="seed", type=int, default=1234)
    a("--label", dest="label", default="")
    a("--query-suffix", "-q", dest="query_suffix", default="")
    a("--store-index", "-s", dest="store_index", action="store_true")
    a("--load-index", "-l", dest="load_index", action="store_true")
    a("--cache", dest="cache", action="store_true")
    a("--routing", dest="routing", action="store_true")
    a("--cache-ratio", dest="cache_ratio", type=int, default=5)
    a("--no-recall", dest="no_recall", action="store_true")
    a("--ip-dist", dest="ip_dist", action="store_true")
    a("--beam-width", "--ef-search", dest="beam_width", type=int, default=0)
    a("--beam-width-construction", "--ef-construction", dest="beam_width_construction", type=int, default=200)
    a("--k", "-k", dest="k", type=int, default=0)
    a("--R", "-m", dest="R", type=int, default=64)
    a("--alpha", dest="alpha", type=float, default=1.2)
    a("--rabitq-bits", dest="rabitq_bits", type=int, default=1)
    a("--search-mode", dest="search_mode", default="exact_gpu")
    a("--insert-workers", dest="insert_workers", type=int, default=0)
    a("--query-workers", dest="query_workers", type=int, default=0)
    a("--insert-coroutines", dest="insert_coroutines", type=int, default=0)
    a("--query-coroutines", dest="query_coroutines", type=int, default=0)
    a("--gpu-device", dest="gpu_device", type=int, default=0)
    a("--gpudirect-rdma", dest="gpudirect_rdma", action="store_true")
    a("--neighbor-cache-mb", dest="neighbor_cache_mb", type=int, default=0)
    a("--gpu-rabitq-cache-mb", dest="gpu_rabitq_cache_mb", type=int, default=0)
    a("--dim", dest="dim", type=int, default=0)
    a("--max-vectors", dest="max_vectors", type=int, default=1_000_000)
    a("--cn-memory", dest="cn_memory", type=int, default=10)
    a("--mn-memory", dest="mn_memory", type=int, default=10)
    return ap


def parse_config(argv) -> ServiceConfig:
    """Parses a compute node's command line and validates it as
    validate_compute_node_options does (configuration.hh:156-198).  The worker
    thread count is not required: the GPU path runs no CPU worker threads."""
    ns = build_parser().parse_args(list(argv))
    fields = {f.name for f in dataclasses.fields(ServiceConfig)}
    cfg = ServiceConfig(**{k: v for k, v in vars(ns).items() if k in fields})
    cfg.search_mode = cfg.search_mode.lower()  # normalize_search_mode (configuration.hh:200-205)
    if cfg.beam_width == 0 or cfg.k == 0 or cfg.dim == 0:
        raise ConfigError("Parameters beam-width (ef-search), k, and dim are required")
    if cfg.store_index and cfg.load_index:
        raise ConfigError("--store-index and --load-index cannot be used in conjunction")
    if (cfg.store_index or cfg.load_index) and not cfg.index_prefix and not cfg.data_path:
        raise ConfigError("--data-path or --index-prefix is required when --load-index or --store-index is set")
    if cfg.cache and cfg.cache_ratio == 0:
        raise ConfigError("If --cache is set, --cache-ratio must be > 0")
    if cfg.search_mode not in SEARCH_MODES:
        raise ConfigError("--search-mode must be exact_gpu or rabitq_gpu")
    if cfg.rabitq_bits not in RABITQ_BITS:
        raise ConfigError("--rabitq-bits must be 1, 2, 4, or 8")
    if cfg.threads:
        if cfg.insert_workers > cfg.threads or cfg.query_workers > cfg.threads:
            raise ConfigError("--insert-workers and --query-workers cannot exceed --threads")
        if cfg.insert_workers > 0 and cfg.query_workers > 0 and cfg.insert_workers + cfg.query_workers != cfg.threads:
            raise ConfigError("--insert-workers + --query-workers must equal --threads when both are set")
    if cfg.insert_coroutines > cfg.coroutines or cfg.query_coroutines > cfg.coroutines:
        raise ConfigError("--insert-coroutines and --query-coroutines cannot exceed --coroutines")
    if cfg.beam_width < cfg.k:
        raise ConfigError("beam_width must be >= k")  # src/vamana/vamana.hh:49
    return cfg


class Service:
    """ComputeService over an HBM-resident index (src/service/compute_service.hh:84-103):
    ``search``, ``insert``, ``load_index``, ``store_index``, ``status``, and the
    ThreadStatistics counters the GPU path produces (``statistics``,
    ``clear_thread_statistics``).  ``load_index``/``store_index`` return
    ``(ok, error_message)`` as the reference returns a bool and fills its
    error string."""

    _COUNTERS = ("processed", "processed_queries", "processed_inserts", "distcomps", "query_distcomps",
                 "build_distcomps", "query_exact_reranks", "visited_neighborlists", "build_overflow_prunes",
                 "query_h2d_bytes", "query_d2h_bytes", "build_h2d_bytes", "build_d2h_bytes")

    def __init__(self, cfg: ServiceConfig, devices=None):
        self.cfg = cfg
        self.devices = tuple(devices) if devices else (cfg.gpu_device,)
        self.index = None
        self.vectors_inserted = 0
        self.stats = dict.fromkeys(self._COUNTERS, 0)
        self.device_ms = {"query": 0.0, "insert": 0.0}
        if cfg.load_index:
            ok, msg = self.load_index(cfg.resolved_index_prefix())
            if not ok:
                raise ConfigError(msg)

    @classmethod
    def from_args(cls, argv, devices=None) -> "Service":
        return cls(parse_config(argv), devices)

    @property
    def mode(self) -> str:
        return self.cfg.search_mode

    def load_index(self, path: str):
        """load_index + maybe_load_rabitq_artifacts (compute_service.cc:280-320, 527-593):
        in rabitq_gpu mode the artifacts' dim and bits must match the flags."""
        from ._lib import DvsError
        from .index import Index

        rabitq = self.cfg.search_mode == "rabitq_gpu"
        try:
            ix = Index(path, devices=self.devices, expect_dim=self.cfg.dim if rabitq else 0,
                       expect_bits=self.cfg.rabitq_bits if rabitq else 0)
        except DvsError as e:
            return False, str(e)
        if ix.dim != self.cfg.dim:
            ix.close()
            return False, f"search dimension mismatch: index {ix.dim}, --dim {self.cfg.dim}"
        if self.index is not None:
            self.index.close()
        self.index = ix
        return True, ""

    def store_index(self, path: str, num_memory_nodes: int = 1):
        """store_index (compute_service.cc:321-337): the current device index,
        inserts included, written in the reference's shard/meta/rotation files."""
        from ._lib import DvsError
        from .index import load_host_index, write_index

        if self.index is None:
            return False, "no index loaded"
        try:
            adj, rec, vec, ids = self.index.download()
            info = self.index.info
            P, c_rot = self._artifacts
            write_index(path, vec, adj, rec, P, c_rot, info.medoid, info.t_const, info.rabitq_bits,
                        num_memory_nodes=num_memory_nodes, beam_width=self.cfg.beam_width_construction,
                        alpha=self.cfg.alpha, metric="ip" if info.metric == 1 else "l2", ids=ids)
        except (DvsError, OSError) as e:
            return False, str(e)
        return True, ""

    def status(self) -> dict:
        """ComputeService::status (compute_service.cc:339-347)."""
        return {"state": "running", "vectors_inserted": self.vectors_inserted, "dimension": self.cfg.dim,
                "threads": self.cfg.threads}

    def search(self, query, k: int):
        """Top-k node ids of one query (ComputeService::search, compute_service.cc:227)."""
        ids, _ = self.search_batch(np.asarray(query, np.float32)[None], k)
        return [int(x) for x in ids[0] if x != 0xFFFFFFFF][:k]

    def search_batch(self, queries, k: int | None = None):
        if self.index is None:
            raise ConfigError("no index loaded")
        q = np.ascontiguousarray(queries, dtype=np.float32)
        if q.ndim != 2 or q.shape[1] != self.cfg.dim:
            raise ValueError("search dimension mismatch")
        kk = min(k or self.cfg.k, self.cfg.k)
        ids, d, st = self.index.search(q, kk, self.cfg.beam_width, self.cfg.search_mode, stats=True)
        n = q.shape[0]
        s = self.stats
        s["processed"] += n
        s["processed_queries"] += n
        s["visited_neighborlists"] += st["expansions"]
        s["query_distcomps"] += st["estimates"]
        s["distcomps"] += st["estimates"]
        s["query_exact_reranks"] += st["reranked"]
        s["query_h2d_bytes"] += q.nbytes
        s["query_d2h_bytes"] += ids.nbytes + d.nbytes
        self.device_ms["query"] += st.get("device_ms", 0.0)
        return ids, d

    def insert(self, batch) -> int:
        """ComputeService::insert (compute_service.cc:152-196): (id, values) items."""
        if self.index is None:
            raise ConfigError("no index loaded")
        if not batch:
            return 0
        for _, values in batch:
            if len(values) != self.cfg.dim:
                raise ValueError("insert dimension mismatch")
        ids = np.array([int(i) for i, _ in batch], np.uint32)
        X = np.array([np.asarray(v, np.float32) for _, v in batch], np.float32)
        st = self.index.insert(X, ids, beam_width_construction=self.cfg.beam_width_construction, alpha=self.cfg.alpha)
        n = int(st["inserted"])
        s = self.stats
        s["processed"] += n
        s["processed_inserts"] += n
        s["build_distcomps"] += st["distances"]
        s["distcomps"] += st["distances"]
        s["visited_neighborlists"] += st["expansions"]
        s["build_overflow_prunes"] += st["full_prunes"]
        s["build_h2d_bytes"] += X.nbytes + ids.nbytes
        self.device_ms["insert"] += st["device_ms"] + st["prune_ms"] + st["reverse_ms"]
        self.vectors_inserted += n
        return n

    def statistics(self) -> dict:
        return dict(self.stats, device_ms=dict(self.device_ms))

    def clear_thread_statistics(self) -> None:
        self.stats = dict.fromkeys(self._COUNTERS, 0)
        self.device_ms = {"query": 0.0, "insert": 0.0}

    def close(self) -> None:
        if self.index is not None:
            self.index.close()
            self.index = None

    @property
    def _artifacts(self):
        """The index's rotation and rotated centroid as they sit on the device."""
        return self.index.artifacts()
