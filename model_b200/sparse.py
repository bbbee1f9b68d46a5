"""Sparse value-table training step over the C ABI (host side).

Mirrors the reference trainer's sparse path (memory_pool_model/train.py):
``fetched_row_grads(aux, probe_grads, layers, pool_size)`` (:146-172) turns
the gradient of each memory layer's read -- taken from the zero probes added
to the reads (model.py:114-115) -- into ``(uniq, rows)``, the distinct
fetched slots and their summed gradients; ``rowwise_adagrad`` applies the
global-norm clip (:378-383) and the row-wise Adagrad update (:396-399) to
the fetched rows only.  Both run in ``libmemlayer.so``; tensors are CUDA
tensors.
"""

from __future__ import annotations

import ctypes as C
import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import _lib as L
from .memory import _workspace, on_stream


def _reads(aux, probe_grads, layers) -> Tuple[List[L.MemlayerRead], list, int, int, int]:
    slots_l = aux["slots"] if isinstance(aux["slots"], (list, tuple)) else [aux["slots"]]
    weights_l = aux["weights"] if isinstance(aux["weights"], (list, tuple)) else [aux["weights"]]
    if not (len(slots_l) == len(weights_l) == len(layers)):
        raise ValueError("one slots / weights entry per memory layer")
    if len(layers) > L.MAX_READS:
        raise ValueError(f"at most {L.MAX_READS} memory layers share a pool")
    keep, reads = [], []
    H = k = d = None
    for layer, sl, w in zip(layers, slots_l, weights_l):
        g = probe_grads[layer]
        for t, name in ((sl, "slots"), (w, "weights"), (g, "probe grad")):
            if not isinstance(t, torch.Tensor) or not t.is_cuda:
                raise TypeError(f"{name} must be a CUDA tensor (no CPU path)")
        H, k = sl.shape[-2], sl.shape[-1]
        d = g.shape[-1]
        sl = sl.to(torch.int32).contiguous()
        w = w.to(torch.float32).contiguous()
        g = g.to(torch.float32).contiguous()
        tokens = sl.numel() // (H * k)
        if w.numel() != sl.numel() or g.numel() != tokens * d:
            raise ValueError("slots, weights and probe grad disagree on the token count")
        keep += [sl, w, g]
        reads.append(L.MemlayerRead(slots=sl.data_ptr(), weights=w.data_ptr(), grad=g.data_ptr(), tokens=tokens))
    return reads, keep, H, k, d


def _config(pool_size: int, H: int, k: int, d: int) -> L.MemlayerConfig:
    n = math.isqrt(pool_size)
    if n * n != pool_size:
        raise ValueError("pool_size must be n_sub_keys ** 2")
    return L.MemlayerConfig(tokens=0, heads=H, n_sub_keys=n, d_key=2, d_value=d, top_k=k, d_model=0,
                            values_dtype=L.F32, routing_noise=0.0, min_temperature=1.0, max_temperature=1.0)


@on_stream
def fetched_row_grads(aux: Dict, probe_grads: Dict, layers: Sequence[int], pool_size: int, *,
                      stream: Optional[torch.cuda.Stream] = None, with_sq_norm: bool = False):
    """train.py:146-172: ``(uniq [cap], rows [cap, d])``, cap = min(fetches,
    pool_size); padding slots equal ``pool_size`` with zero rows.
    ``aux["slots"]`` / ``aux["weights"]`` hold one entry per layer of
    ``layers``; ``probe_grads[layer]`` is dL/d(read output) [..., d]."""
    reads, keep, H, k, d = _reads(aux, probe_grads, layers)
    device = keep[0].device
    F = sum(r.tokens for r in reads) * H * k
    cfg = _config(pool_size, H, k, d)
    cap = min(F, pool_size)
    uniq = torch.empty(cap, dtype=torch.int32, device=device)
    rows = torch.empty(cap, d, dtype=torch.float32, device=device)
    n_unique = torch.empty(1, dtype=torch.int32, device=device)
    sq = torch.empty(1, dtype=torch.float32, device=device)
    nb = C.c_size_t()
    L.check(L.lib().memlayer_rowgrad_workspace_size(C.byref(cfg), F, C.byref(nb)), "memlayer_rowgrad_workspace_size")
    ws = _workspace(nb.value, device)
    arr = (L.MemlayerRead * len(reads))(*reads)
    s = (stream or torch.cuda.current_stream(device)).cuda_stream
    L.check(L.lib().memlayer_fetched_row_grads(C.byref(cfg), arr, len(reads), uniq.data_ptr(), rows.data_ptr(),
                                               n_unique.data_ptr(), sq.data_ptr(), ws.data_ptr(), nb.value, s),
            "memlayer_fetched_row_grads")
    out = (uniq, rows)
    if with_sq_norm:
        out = out + (n_unique, sq, ws, cfg)
    return out


@on_stream
def rowwise_adagrad(values: torch.Tensor, accum: torch.Tensor, aux: Dict, probe_grads: Dict,
                    layers: Sequence[int], *, lr: float, grad_clip: float,
                    rest_sq_norm: Optional[torch.Tensor] = None, stream: Optional[torch.cuda.Stream] = None,
                    check: bool = False) -> Dict[str, torch.Tensor]:
    """Clip by the global norm of (rest, row grads) and apply row-wise
    Adagrad to the fetched rows of ``values`` / ``accum`` in place
    (train.py:378-383, 396-399).  Returns {"clip_scale", "n_unique"}."""
    if values.dtype != torch.float32 or not values.is_cuda or not values.is_contiguous():
        raise TypeError("values must be a contiguous float32 CUDA tensor")
    if accum.dtype != torch.float32 or accum.numel() != values.shape[0] or not accum.is_contiguous():
        raise TypeError("accum must be a contiguous float32 tensor with one entry per row")
    reads, keep, H, k, d = _reads(aux, probe_grads, layers)
    device = values.device
    F = sum(r.tokens for r in reads) * H * k
    cfg = _config(values.shape[0], H, k, d)
    scale = torch.empty(1, dtype=torch.float32, device=device)
    n_unique = torch.empty(1, dtype=torch.int32, device=device)
    rest = None if rest_sq_norm is None else rest_sq_norm.to(device, torch.float32).reshape(1).contiguous()
    a = L.MemlayerAdagradArgs(values=values.data_ptr(), accum=accum.data_ptr(), lr=float(lr),
                              grad_clip=float(grad_clip), rest_sq_norm=None if rest is None else rest.data_ptr(),
                              clip_scale=scale.data_ptr(), n_unique=n_unique.data_ptr())
    nb = C.c_size_t()
    L.check(L.lib().memlayer_rowgrad_workspace_size(C.byref(cfg), F, C.byref(nb)), "memlayer_rowgrad_workspace_size")
    ws = _workspace(nb.value, device)
    arr = (L.MemlayerRead * len(reads))(*reads)
    s = (stream or torch.cuda.current_stream(device)).cuda_stream
    L.check(L.lib().memlayer_row_adagrad(C.byref(cfg), arr, len(reads), C.byref(a), ws.data_ptr(), nb.value, s),
            "memlayer_row_adagrad")
    if check:
        code = L.device_status(cfg, ws.data_ptr(), s)
        if code:
            raise L.DeviceError(f"device status {code}: {L.DEVICE_ERRORS.get(code, 'unknown')}")
    return {"clip_scale": scale, "n_unique": n_unique}


class ShardedRowUpdate:
    """One rank's owner-sharded row update over a row-update communicator
    (``model_b200.shard.connect(cfg, n_reads=...)``): ``values`` / ``accum``
    are this rank's rows (slot s on rank s % world, local row s / world);
    ``aux`` / ``probe_grads`` hold this rank's reads.  ``run(phases)`` runs
    ROUTE (local merge + push), GATHER (owner merge) and REDUCE (clip +
    Adagrad) -- every rank must run every phase of a step."""

    def __init__(self, comm, values: torch.Tensor, accum: torch.Tensor, aux: Dict, probe_grads: Dict,
                 layers: Sequence[int], *, lr: float, grad_clip: float,
                 rest_sq_norm: Optional[torch.Tensor] = None):
        if values.dtype != torch.float32 or not values.is_cuda or not values.is_contiguous():
            raise TypeError("values must be a contiguous float32 CUDA tensor")
        if accum.dtype != torch.float32 or accum.numel() != values.shape[0] or not accum.is_contiguous():
            raise TypeError("accum must be a contiguous float32 tensor with one entry per local row")
        self.comm = comm
        reads, self._keep, H, k, d = _reads(aux, probe_grads, layers)
        self.device = values.device
        self.cfg = _config(comm.cfg.n_sub_keys ** 2, H, k, d)
        F = sum(r.tokens for r in reads) * H * k
        self.scale = torch.empty(1, dtype=torch.float32, device=self.device)
        self.n_unique = torch.empty(1, dtype=torch.int32, device=self.device)
        self._rest = None if rest_sq_norm is None else rest_sq_norm.to(self.device, torch.float32).reshape(1).contiguous()
        self.args = L.MemlayerAdagradArgs(values=values.data_ptr(), accum=accum.data_ptr(), lr=float(lr),
                                          grad_clip=float(grad_clip),
                                          rest_sq_norm=None if self._rest is None else self._rest.data_ptr(),
                                          clip_scale=self.scale.data_ptr(), n_unique=self.n_unique.data_ptr())
        nb = C.c_size_t()
        L.check(L.lib().memlayer_shard_rowgrad_workspace_size(comm.handle, F, C.byref(nb)),
                "memlayer_shard_rowgrad_workspace_size")
        self.nbytes = nb.value
        self.ws = _workspace(nb.value, self.device)
        self._arr = (L.MemlayerRead * len(reads))(*reads)
        self._n = len(reads)
        self._values, self._accum = values, accum

    def run(self, phases: int = L.PHASE_ALL, stream: Optional[torch.cuda.Stream] = None) -> None:
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        L.check(L.lib().memlayer_row_adagrad_sharded(C.byref(self.cfg), self._arr, self._n, C.byref(self.args),
                                                     self.comm.handle, phases, self.ws.data_ptr(), self.nbytes, s),
                "memlayer_row_adagrad_sharded")

    def check(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        code = L.device_status(self.cfg, self.ws.data_ptr(), s)
        if code:
            raise L.DeviceError(f"device status {code}: {L.DEVICE_ERRORS.get(code, 'unknown')}")

    def result(self) -> Dict[str, torch.Tensor]:
        return {"clip_scale": self.scale, "n_unique": self.n_unique}


@on_stream
def sharded_rowwise_adagrad(values: torch.Tensor, accum: torch.Tensor, aux: Dict, probe_grads: Dict,
                            layers: Sequence[int], comm, *, lr: float, grad_clip: float,
                            rest_sq_norm: Optional[torch.Tensor] = None, stream: Optional[torch.cuda.Stream] = None,
                            check: bool = False) -> Dict[str, torch.Tensor]:
    """The row-sharded counterpart of :func:`rowwise_adagrad` (train.py:175-206
    merge + :378-399 clip and update): all three phases on this rank.
    Returns {"clip_scale" (global), "n_unique" (rows this rank updated)}."""
    up = ShardedRowUpdate(comm, values, accum, aux, probe_grads, layers, lr=lr, grad_clip=grad_clip,
                          rest_sq_norm=rest_sq_norm)
    up.run(L.PHASE_ALL, stream)
    if check:
        up.check(stream)
    return up.result()
