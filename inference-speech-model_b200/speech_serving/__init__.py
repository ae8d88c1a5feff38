"""B200-native speech decode engine: the decode-attention hot path of a Whisper-class
serving engine (paged self-attention, cross-attention, K/V append, block gather and the
handoff cross-KV projection) as sm_100a kernels behind a C ABI, with the Python operator
surface of the original engine (scheduler, cache managers, graph decode slots)."""
import os

os.environ.setdefault("USE_TF", "0")
os.environ.setdefault("TRANSFORMERS_NO_TF", "1")

from . import ops  # noqa: E402,F401
from .block_manager import BlockManager  # noqa: E402,F401
from .dual_cache_manager import DualCacheManager  # noqa: E402,F401
from .encoder_block_manager import EncoderBlockManager  # noqa: E402,F401
from .memory_guard import MemoryGuard  # noqa: E402,F401
