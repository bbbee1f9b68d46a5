"""Sub-key maintenance of the training step over the C ABI (host side).

Mirrors the reference's ``key_diversity_loss(sub_keys)``
(memory_pool_model/memory.py:230-240; the trainer adds
``key_diversity_coef * loss``, train.py:327-329) and ``revive_dead_keys(
sub_keys, subkey_usage, queries, rng, threshold, noise=0.05)``
(memory.py:243-281, called from train.py:486-509, which also clears the
optimiser moments of revived keys).  The reference draws the revival's
token picks and noise from ``rng`` inside the call; here the caller passes
the draws (``pick`` [H, 2, n] int, ``noise`` [H, 2, n, half]), or a
``torch.Generator`` from which :func:`revive_dead_keys` draws them on the
device.  Both run in ``libmemlayer.so``; tensors are CUDA tensors.
"""

from __future__ import annotations

import ctypes as C
from typing import Optional, Sequence, Tuple

import torch

from . import _lib as L
from .memory import _workspace, on_stream


def _config(sub_keys: torch.Tensor) -> L.MemlayerConfig:
    if not isinstance(sub_keys, torch.Tensor) or not sub_keys.is_cuda:
        raise TypeError("sub_keys must be a CUDA tensor (no CPU path)")
    if sub_keys.dim() != 4 or sub_keys.shape[1] != 2:
        raise ValueError("sub_keys must be [H, 2, n, d_key / 2]")
    H, _, n, half = sub_keys.shape
    return L.MemlayerConfig(tokens=0, heads=H, n_sub_keys=n, d_key=2 * half, d_value=4, top_k=1, d_model=0,
                            values_dtype=L.F32, routing_noise=0.0, min_temperature=1.0, max_temperature=1.0)


def _f32(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor (no CPU path)")
    return t.to(torch.float32).contiguous()


@on_stream
def key_diversity_loss(sub_keys: torch.Tensor, *, grad: bool = False, grad_scale: float = 1.0,
                       stream: Optional[torch.cuda.Stream] = None):
    """memory.py:230-240: mean squared off-diagonal cosine of the unit
    sub-keys inside each codebook (a 0-dim float32 tensor).  With
    ``grad=True`` returns ``(loss, grad_scale * d loss / d sub_keys)``."""
    cfg = _config(sub_keys)
    x = _f32(sub_keys, "sub_keys")
    device = x.device
    loss = torch.empty((), dtype=torch.float32, device=device)
    g = torch.empty_like(x) if grad else None
    nb = C.c_size_t()
    L.check(L.lib().memlayer_key_diversity_workspace_size(C.byref(cfg), C.byref(nb)),
            "memlayer_key_diversity_workspace_size")
    ws = _workspace(nb.value, device)
    s = (stream or torch.cuda.current_stream(device)).cuda_stream
    L.check(L.lib().memlayer_key_diversity(C.byref(cfg), x.data_ptr(), loss.data_ptr(),
                                           None if g is None else g.data_ptr(), float(grad_scale), ws.data_ptr(),
                                           nb.value, s), "memlayer_key_diversity")
    return (loss, g) if grad else loss


@on_stream
def revive_dead_keys(sub_keys: torch.Tensor, subkey_usage: torch.Tensor, queries: torch.Tensor,
                     threshold: float, noise: float = 0.05, *, pick: Optional[torch.Tensor] = None,
                     normal: Optional[torch.Tensor] = None, generator: Optional[torch.Generator] = None,
                     moments: Sequence[torch.Tensor] = (), stream: Optional[torch.cuda.Stream] = None,
                     ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """memory.py:243-281: returns ``(new_sub_keys, new_subkey_usage, dead)``.

    ``queries`` [M, H, 2, half] are unit query halves (``aux["queries"]``).
    ``pick`` [H, 2, n] and ``normal`` [H, 2, n, half] are the random draws
    (token index, standard normal); missing ones are drawn on the device from
    ``generator``.  Each tensor of ``moments`` (optimiser state shaped like
    sub_keys, float32, contiguous) has its revived rows zeroed in place
    (train.py:497-509).
    """
    cfg = _config(sub_keys)
    H, _, n, half = sub_keys.shape
    device = sub_keys.device
    keys = _f32(sub_keys, "sub_keys").clone()
    usage = _f32(subkey_usage, "subkey_usage").clone()
    q = _f32(queries, "queries")
    if usage.shape != (H, 2, n):
        raise ValueError("subkey_usage must be [H, 2, n]")
    if q.dim() != 4 or tuple(q.shape[1:]) != (H, 2, half) or q.shape[0] < 1:
        raise ValueError("queries must be [M >= 1, H, 2, d_key / 2]")
    if pick is None:
        pick = torch.randint(0, q.shape[0], (H, 2, n), device=device, generator=generator)
    if normal is None:
        normal = torch.randn(H, 2, n, half, device=device, generator=generator)
    pick = pick.to(device, torch.int32).contiguous()
    normal = _f32(normal, "normal")
    if pick.shape != (H, 2, n) or normal.shape != keys.shape:
        raise ValueError("pick must be [H, 2, n] and normal shaped like sub_keys")
    if len(moments) > 2:
        raise ValueError("at most two optimiser moments")
    for m in moments:
        if m.dtype != torch.float32 or m.shape != keys.shape or not m.is_contiguous() or m.device != device:
            raise TypeError("moments must be contiguous float32 tensors shaped like sub_keys")
    mom = [m.data_ptr() for m in moments] + [None] * (2 - len(moments))
    dead = torch.empty(H, 2, n, dtype=torch.int32, device=device)
    a = L.MemlayerReviveArgs(sub_keys=keys.data_ptr(), usage=usage.data_ptr(), queries=q.data_ptr(),
                             query_tokens=q.shape[0], pick=pick.data_ptr(), noise=normal.data_ptr(),
                             threshold=float(threshold), noise_scale=float(noise), dead=dead.data_ptr(),
                             moment0=mom[0], moment1=mom[1])
    s = (stream or torch.cuda.current_stream(device)).cuda_stream
    L.check(L.lib().memlayer_revive_dead_keys(C.byref(cfg), C.byref(a), s), "memlayer_revive_dead_keys")
    return keys, usage, dead.bool()
