"""Re-export of speech_serving.block_manager.BlockManager (reference paged_kv_cache/block_manager.py:9)."""
from speech_serving.block_manager import BlockManager

__all__ = ["BlockManager"]
