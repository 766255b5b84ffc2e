"""NumPy interface for Quiver approximate nearest neighbour search (B200 engine)."""

from .index import IndexQuiver, QuiverError

__all__ = ["IndexQuiver", "QuiverError"]
__version__ = "0.1.0"
