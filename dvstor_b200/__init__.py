"""B200-native DVSTOR `rabitq_gpu` query path.

The compute lives in libdvs_b200.so (C ABI, include/dvs_b200.h): a persistent
sm_100a kernel that runs Vamana beam search with RaBitQ estimates and an exact
rerank on an HBM-resident index read from the reference's offline formats.
This package is the host-side mirror of the reference's query interface.
"""
from ._lib import DvsError, EMPTY, lib
from .index import ComputeService, Index, load_host_index, write_index

__all__ = ["ComputeService", "DvsError", "EMPTY", "Index", "lib", "load_host_index", "write_index"]
