"""quiver_b200 -- B200-native engine for Quiver's query hot path.

Graph beam search over a Vamana/DiskANN-layout index, scored by PQ
asymmetric distance and finished with an exact-L2 top-k, run by a
persistent sm_100a kernel behind the C ABI in ``include/quiver_b200.h``.
"""
from ._lib import NativeLibraryMissing
from .engine import Engine, QuiverEngineError, SearchParams
from .index import IndexQuiver, QuiverError

__all__ = ["Engine", "SearchParams", "QuiverEngineError", "NativeLibraryMissing", "IndexQuiver", "QuiverError"]
__version__ = "0.1.0"
