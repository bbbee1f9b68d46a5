"""On-disk format of the value table and its optimiser state.

The reference keeps the pool's arrays as ``.npy`` files in one directory
(memory_pool_model/host_pool.py:90-108: ``values.npy`` [n_slots, dim] in the
table's dtype, ``m.npy`` / ``v.npy`` [n_slots, dim] float32 for Adam,
``acc.npy`` [n_slots] float32 for row-wise Adagrad) and snapshots them by
writing ``<key>.tmp.npy`` and renaming it over ``<key>.npy``
(host_pool.py:175-188).  This module reads and writes the same files for the
row-sharded table of this package: rank ``r`` of ``world`` holds slots
``s % world == r`` as local rows ``s // world``, so each rank writes and
reads the strided rows ``r::world`` of the shared files.  A snapshot written
at one world size loads at any other, and the files load with the
reference's ``HostPool.load`` / ``np.load``.

Rows move between the device and the file in chunks through a pinned host
buffer (one copy per chunk on the caller's stream).
"""

from __future__ import annotations

import os
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

KEYS = ("values", "m", "v", "acc")
_CHUNK_BYTES = 64 << 20

_NP = {torch.float32: np.float32, torch.float16: np.float16}


def _np_dtype(t: torch.Tensor):
    if t.dtype not in _NP:
        raise TypeError(f"{t.dtype} has no .npy counterpart in the reference's format (float32 / float16)")
    return _NP[t.dtype]


def _barrier(group):
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        dist.barrier(group)


def _gather_problems(problem: Optional[str], group) -> List[str]:
    """Every rank's argument problem (None when fine), on every rank."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()):
        return [problem] if problem else []
    out: List[Optional[str]] = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, problem, group=group)
    return [f"rank {r}: {p}" for r, p in enumerate(out) if p]


def _local_rows(n_slots: int, rank: int, world: int) -> int:
    return (n_slots - rank + world - 1) // world if n_slots > rank else 0


def _write_rows(mm: np.ndarray, local: torch.Tensor, rank: int, world: int) -> None:
    """mm[rank::world] = local, chunk by chunk through pinned memory."""
    rows = local.shape[0]
    if rows == 0:
        return
    row_bytes = max(local[0].numel() * local.element_size(), 1)
    step = max(1, _CHUNK_BYTES // row_bytes)
    pinned = torch.empty((min(step, rows),) + tuple(local.shape[1:]), dtype=local.dtype,
                         pin_memory=local.is_cuda)
    view = mm[rank::world]
    for i0 in range(0, rows, step):
        i1 = min(i0 + step, rows)
        buf = pinned[: i1 - i0]
        buf.copy_(local[i0:i1], non_blocking=local.is_cuda)
        if local.is_cuda:
            torch.cuda.current_stream(local.device).synchronize()
        view[i0:i1] = buf.numpy()


def _read_rows(mm: np.ndarray, out: torch.Tensor, rank: int, world: int) -> None:
    """out = mm[rank::world], chunk by chunk through pinned memory."""
    rows = out.shape[0]
    if rows == 0:
        return
    row_bytes = max(out[0].numel() * out.element_size(), 1)
    step = max(1, _CHUNK_BYTES // row_bytes)
    pinned = torch.empty((min(step, rows),) + tuple(out.shape[1:]), dtype=out.dtype, pin_memory=out.is_cuda)
    view = mm[rank::world]
    for i0 in range(0, rows, step):
        i1 = min(i0 + step, rows)
        buf = pinned[: i1 - i0]
        buf.numpy()[...] = view[i0:i1]
        out[i0:i1].copy_(buf, non_blocking=out.is_cuda)
        if out.is_cuda:
            torch.cuda.current_stream(out.device).synchronize()   # the pinned buffer is reused


def save_table(dest: str, arrays: Dict[str, torch.Tensor], n_slots: int, rank: int = 0, world: int = 1,
               group=None) -> None:
    """Snapshot this rank's rows into ``dest/<key>.npy`` (host_pool.py:175-182).

    ``arrays`` maps keys of ``KEYS`` to this rank's local rows ([rows, dim]
    for values / m / v, [rows] for acc), rows = slots ``rank::world``.
    Collective when ``world > 1`` (torch.distributed): rank 0 creates each
    ``<key>.tmp.npy``, every rank writes its rows, rank 0 renames the file
    over ``<key>.npy`` once all ranks have flushed.
    """
    problem = None
    for key, t in arrays.items():
        if key not in KEYS:
            problem = f"unknown table array {key!r}; expected one of {KEYS}"
        elif t.shape[0] != _local_rows(n_slots, rank, world):
            problem = (f"{key}: {t.shape[0]} local rows, expected {_local_rows(n_slots, rank, world)} "
                       f"for rank {rank} of {world}")
        elif (key == "acc") != (t.dim() == 1):
            problem = f"{key}: acc is [rows], the others [rows, dim]"
        if problem:
            break
    # every rank learns of any rank's bad arguments before the first barrier,
    # so all raise together instead of the others waiting in a collective
    problems = _gather_problems(problem, group)
    if problems:
        raise ValueError("; ".join(problems))
    if rank == 0:
        os.makedirs(dest, exist_ok=True)
    _barrier(group)
    for key in KEYS:
        if key not in arrays:
            continue
        t = arrays[key]
        shape = (n_slots,) + tuple(t.shape[1:])
        tmp = os.path.join(dest, f"{key}.tmp.npy")
        if rank == 0:
            np.lib.format.open_memmap(tmp, mode="w+", dtype=_np_dtype(t), shape=shape).flush()
        _barrier(group)
        mm = np.lib.format.open_memmap(tmp, mode="r+")
        if mm.shape != shape or mm.dtype != _np_dtype(t):
            raise ValueError(f"{tmp}: {mm.shape} {mm.dtype}, expected {shape} {_np_dtype(t)}")
        _write_rows(mm, t.detach(), rank, world)
        mm.flush()
        del mm
        _barrier(group)
        if rank == 0:
            os.replace(tmp, os.path.join(dest, f"{key}.npy"))
        _barrier(group)


def load_table(src: str, keys: Sequence[str], rank: int = 0, world: int = 1,
               device: Optional[torch.device] = None, dtype: Optional[torch.dtype] = None) -> Dict[str, torch.Tensor]:
    """This rank's rows of ``src/<key>.npy`` (host_pool.py:184-188), any world
    size: {key: tensor [rows, dim] or [rows]}.  ``dtype`` converts values
    (e.g. a float32 file into a float16 table); m / v / acc stay float32.
    Missing files are skipped, as the reference's ``load`` does."""
    out: Dict[str, torch.Tensor] = {}
    for key in keys:
        if key not in KEYS:
            raise ValueError(f"unknown table array {key!r}; expected one of {KEYS}")
        f = os.path.join(src, f"{key}.npy")
        if not os.path.exists(f):
            continue
        mm = np.load(f, mmap_mode="r")
        rows = _local_rows(mm.shape[0], rank, world)
        np_dt = mm.dtype
        if np_dt not in (np.dtype(np.float32), np.dtype(np.float16)):
            raise TypeError(f"{f}: dtype {np_dt} is not float32 / float16")
        file_dt = torch.float32 if np_dt == np.float32 else torch.float16
        t = torch.empty((rows,) + tuple(mm.shape[1:]), dtype=file_dt, device=device)
        _read_rows(mm, t, rank, world)
        if key == "values" and dtype is not None and dtype != file_dt:
            t = t.to(dtype)
        out[key] = t
    return out


def open_table(path: str, n_slots: int, dim: int, dtype=np.float32, optimizer: Optional[str] = "rowwise_adagrad",
               seed: int = 0) -> Dict[str, np.ndarray]:
    """The reference's memmap layout of a live host pool (host_pool.py:90-108):
    creates missing files (values initialised normal(0, dim**-0.5) in chunks,
    optimiser state zero) and reopens existing ones, checking their shapes."""
    os.makedirs(path, exist_ok=True)
    specs = [("values", dtype, (n_slots, dim))]
    if optimizer == "adam":
        specs += [("m", np.float32, (n_slots, dim)), ("v", np.float32, (n_slots, dim))]
    elif optimizer == "rowwise_adagrad":
        specs += [("acc", np.float32, (n_slots,))]
    elif optimizer is not None:
        raise ValueError(f"unknown pool optimizer {optimizer!r}")
    arrs = {}
    for key, dt, shape in specs:
        f = os.path.join(path, f"{key}.npy")
        fresh = not os.path.exists(f)
        a = np.lib.format.open_memmap(f, mode="w+" if fresh else "r+", dtype=dt, shape=shape)
        if not fresh and a.shape != shape:
            raise ValueError(f"{f} has shape {a.shape}, expected {shape}")
        if fresh and key == "values":
            rng = np.random.default_rng(seed)
            for s in range(0, n_slots, 1 << 18):
                e = min(s + (1 << 18), n_slots)
                a[s:e] = (rng.standard_normal((e - s, dim)) * dim ** -0.5).astype(dt)
        arrs[key] = a
    return arrs
