"""``from paged_kv_cache.block_manager import BlockManager`` compatibility import, as the
reference provides (paged_kv_cache/__init__.py:22)."""
from speech_serving.block_manager import BlockManager

__all__ = ["BlockManager"]
