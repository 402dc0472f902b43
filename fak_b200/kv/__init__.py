"""KV cache management: refcounted page pool and radix-tree prefix cache."""
from .radix import OutOfPages, PagePool, RadixCache

__all__ = ["OutOfPages", "PagePool", "RadixCache"]
