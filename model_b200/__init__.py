"""B200 (sm_100a) product-key memory layer of KumarDev7/model.

``MemoryPool`` / ``MemoryLayer`` mirror the reference's Flax module and its
caller block; every step runs in the CUDA library ``libmemlayer.so`` behind
the C ABI of ``include/memlayer.h``.
"""

from .memory import MemoryLayer, MemoryPool  # noqa: F401

__all__ = ["MemoryPool", "MemoryLayer"]
