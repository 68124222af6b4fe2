"""helix_online_kv -- compressed KV cache with B200 (sm_100a) CUDA kernels.

Same public surface as the reference package (echo313unfolding/helix-online-kv,
helix_online_kv/__init__.py:5-10), plus ``CompressedKVCache`` (imported on
first access, as it pulls in transformers) and the batched device API
``cdc03.CDC03Store``.
"""

__version__ = "0.1.0"

from .config import OnlineKVConfig
from .codebook import OnlineCodebook
from .vector_codebook import VectorCodebook
from .product_codebook import ProductCodebook
from .layer_state import KVLayerState
from .aging_policy import AgingPolicy


def __getattr__(name):
    if name == "CompressedKVCache":
        from .compressed_cache import CompressedKVCache
        return CompressedKVCache
    raise AttributeError(f"module 'helix_online_kv' has no attribute {name!r}")
