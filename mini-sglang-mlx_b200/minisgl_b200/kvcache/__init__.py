from .pool import MHAKVCache

__all__ = ["MHAKVCache"]
