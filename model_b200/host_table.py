"""Value table in page-locked host memory: the read side of the reference's
host tier (memory_pool_model/host_pool.py:62-127 HostPool, :206-220 fetch).

``HostTable(n_slots, dim)`` keeps ``values`` [n_slots, dim] (float16 or
float32) in pinned host RAM, which the GPU reads directly; registered by
name like the reference's pools (host_pool.py:25,54), so that
``MemoryPool(host_pool=name)`` serves reads from it through
``memlayer_pool_forward_host_table`` (distinct rows fetched once per call by
the GPU).  The table loads from and saves to the reference's ``values.npy``
layout (``model_b200.table_io``).  Pools larger than host RAM (the
reference's SSD memmaps) are not served: the GPU reads only page-locked
memory, and GPUDirect Storage is not available here.
"""

from __future__ import annotations

import os
import uuid
from typing import Dict, Optional

import numpy as np
import torch

_REGISTRY: Dict[str, "HostTable"] = {}
_INIT_CHUNK = 1 << 18    # rows initialised per chunk (host_pool.py:29)
_NP = {torch.float16: np.float16, torch.float32: np.float32}


def get(name: str) -> "HostTable":
    if name not in _REGISTRY:
        raise KeyError(f"no host table named {name!r}")
    return _REGISTRY[name]


class HostTable:
    """values [n_slots, dim] in page-locked host memory.  ``path`` names a
    directory holding ``values.npy`` (loaded when present); otherwise the
    rows are drawn like the reference's fresh pool, normal(0, dim**-0.5) from
    ``numpy.random.default_rng(seed)`` in chunks (host_pool.py:100-105)."""

    def __init__(self, n_slots: int, dim: int, path: Optional[str] = None, dtype: torch.dtype = torch.float16,
                 seed: int = 0, name: Optional[str] = None):
        if dtype not in _NP:
            raise TypeError("host tables hold float16 or float32 rows")
        if not torch.cuda.is_available():
            raise RuntimeError("a host table is read by the GPU: CUDA is required")
        self.n_slots, self.dim, self.path = n_slots, dim, path
        self.name = name or f"pool-{uuid.uuid4().hex[:8]}"
        self.values = torch.empty(n_slots, dim, dtype=dtype, pin_memory=True)
        arr = self.values.numpy()
        f = os.path.join(path, "values.npy") if path else None
        if f and os.path.exists(f):
            src = np.load(f, mmap_mode="r")
            if src.shape != (n_slots, dim):
                raise ValueError(f"{f} has shape {src.shape}, expected {(n_slots, dim)}")
            for s in range(0, n_slots, _INIT_CHUNK):
                e = min(s + _INIT_CHUNK, n_slots)
                arr[s:e] = src[s:e]
        else:
            rng = np.random.default_rng(seed)
            for s in range(0, n_slots, _INIT_CHUNK):
                e = min(s + _INIT_CHUNK, n_slots)
                arr[s:e] = (rng.standard_normal((e - s, dim)) * dim ** -0.5).astype(_NP[dtype])
        _REGISTRY[self.name] = self

    def nbytes(self) -> int:
        return self.values.numel() * self.values.element_size()

    def save(self, dest: str) -> None:
        """``dest/values.npy`` in the reference's snapshot layout (host_pool.py:175-182)."""
        from .table_io import save_table
        save_table(dest, {"values": self.values}, self.n_slots)

    def close(self) -> None:
        _REGISTRY.pop(self.name, None)
