"""swann_b200: SWANN's multi-branch graph search and exact-sweep graph build on B200.

A drop-in for the reference package `swann` (geniussyn/SWANN): the same
`Index`, `SearchConfig` and `overflow_guard`, with the search and build running
as hand-written sm_100a kernels in libswann_b200.so.

    import swann_b200 as swann
    index = swann.Index.build(X, metric="ip")
    ids, dist = index.search(Q, k=10)
"""
from ._engine import overflow_guard
from .index import Index, SearchConfig

__all__ = ["Index", "SearchConfig", "overflow_guard"]
__version__ = "0.1.0"
