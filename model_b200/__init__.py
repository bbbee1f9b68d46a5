"""B200 (sm_100a) product-key memory layer of KumarDev7/model.

``MemoryPool`` / ``MemoryLayer`` mirror the reference's Flax module and its
caller block, ``MemoryPoolLM`` / ``Generator`` the language model and its
decoder around them; every step runs in the CUDA library ``libmemlayer.so`` behind
the C ABI of ``include/memlayer.h``.
"""

from .memory import MemoryLayer, MemoryPool  # noqa: F401
from .model import Generator, MemoryPoolLM, ModelConfig  # noqa: F401

__all__ = ["MemoryPool", "MemoryLayer", "MemoryPoolLM", "ModelConfig", "Generator"]
