"""Row-sharded value table over the GPUs of one node (host side).

The reference replicates every parameter, the value table included, on each
device of its data-parallel mesh (memory_pool_model/train.py:229-236,267);
this module serves tables larger than one GPU.  Slot ``s`` lives on rank
``s % world`` as local row ``s // world``; sub-keys and the Dense kernels
are replicated.  Each rank routes its own tokens, the owners gather their
rows and return one float32 partial row per (token, owner) over NVLink, and
the token owner adds the partials in rank order (see
``model_b200/csrc/shard.cu``).

One process per GPU: :func:`connect` creates this rank's communicator and
maps every peer's buffer through CUDA IPC handles exchanged with
``torch.distributed.all_gather_object``.  :class:`ShardedCall` also runs the
three phases separately, which lets one process drive several emulated ranks
on one GPU (tests).
"""

from __future__ import annotations

import ctypes as C
import math
from typing import Dict, List, Optional, Sequence

import torch

from . import _lib as L
from .memory import MemoryLayer, MemoryPool, _cuda_f32, _ptr, _raise_device_status, _workspace, on_stream


def shard_rows(pool_size: int, rank: int, world: int) -> int:
    """Rows held by ``rank``: slots s < pool_size with s % world == rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    return max(0, (pool_size - rank + world - 1) // world)


def shard_values(values: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's local rows of a full table (row s // world of rank s % world)."""
    return values[rank::world].contiguous()


def owner_of(slots: torch.Tensor, world: int):
    """(owner rank, local row) of each slot id."""
    return slots % world, slots // world


class ShardComm:
    """This rank's communicator (memlayer_shard_comm) for one set of shapes."""

    def __init__(self, cfg: L.MemlayerConfig, rank: int, world: int, n_reads: Optional[int] = None):
        """``n_reads`` given: a row-update communicator
        (memlayer_shard_comm_create_rowgrad) for that many memory layers."""
        self.rank, self.world = rank, world
        self.cfg = cfg
        self.n_reads = n_reads
        h = C.c_void_p()
        if n_reads is None:
            L.check(L.lib().memlayer_shard_comm_create(C.byref(cfg), rank, world, C.byref(h)),
                    "memlayer_shard_comm_create")
        else:
            L.check(L.lib().memlayer_shard_comm_create_rowgrad(C.byref(cfg), n_reads, rank, world, C.byref(h)),
                    "memlayer_shard_comm_create_rowgrad")
        self.handle = h
        dev, nbytes = C.c_int32(), C.c_size_t()
        L.check(L.lib().memlayer_shard_comm_info(h, None, None, C.byref(dev), C.byref(nbytes)),
                "memlayer_shard_comm_info")
        self.device, self.nbytes = dev.value, nbytes.value
        if self.device != torch.cuda.current_device():
            self.close()
            raise RuntimeError(f"library device {self.device} != torch current device "
                               f"{torch.cuda.current_device()}: call torch.cuda.set_device first")

    def ipc_handle(self) -> bytes:
        buf = (C.c_char * L.IPC_HANDLE_BYTES)()
        L.check(L.lib().memlayer_shard_comm_ipc_handle(self.handle, buf), "memlayer_shard_comm_ipc_handle")
        return bytes(buf)

    def open_peers(self, handles: Sequence[bytes]) -> None:
        if len(handles) != self.world or any(len(h) != L.IPC_HANDLE_BYTES for h in handles):
            raise ValueError(f"need {self.world} handles of {L.IPC_HANDLE_BYTES} bytes")
        blob = b"".join(handles)
        L.check(L.lib().memlayer_shard_comm_open_peers(self.handle, blob), "memlayer_shard_comm_open_peers")

    def set_peer(self, other: "ShardComm") -> None:
        L.check(L.lib().memlayer_shard_comm_set_peer(self.handle, other.rank, other.handle),
                "memlayer_shard_comm_set_peer")

    def set_wait_budget(self, seconds: float) -> None:
        """Budget of each wait on another rank (default 2 s): a wait that
        runs out leaves status 31-36 in the call's workspace instead of a hang."""
        L.check(L.lib().memlayer_shard_comm_set_wait_budget(self.handle, int(round(seconds * 1e9))),
                "memlayer_shard_comm_set_wait_budget")

    def close(self) -> None:
        if self.handle:
            L.check(L.lib().memlayer_shard_comm_destroy(self.handle), "memlayer_shard_comm_destroy")
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def exchange_handles(handle: bytes, group=None) -> List[bytes]:
    """All ranks' IPC handles in rank order (any torch.distributed backend)."""
    import torch.distributed as dist

    out: List[Optional[bytes]] = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return [bytes(h) for h in out]


def connect(cfg: L.MemlayerConfig, group=None, n_reads: Optional[int] = None) -> ShardComm:
    """Create this rank's communicator (a row-update one with ``n_reads``)
    and map every peer's buffer.  Collective over ``group``: every rank calls
    it with the same shapes."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    shapes: List[Optional[tuple]] = [None] * world
    mine = tuple(getattr(cfg, f) for f, _ in cfg._fields_)
    dist.all_gather_object(shapes, mine, group=group)
    if any(s != mine for s in shapes):
        raise ValueError("every rank must create its communicator with the same config")
    comm = ShardComm(cfg, dist.get_rank(group), world, n_reads)
    comm.open_peers(exchange_handles(comm.ipc_handle(), group))
    dist.barrier(group)
    return comm


def emulated_comms(cfg: L.MemlayerConfig, world: int, n_reads: Optional[int] = None) -> List[ShardComm]:
    """``world`` communicators in this process on the current device, wired to
    each other directly (no IPC): for driving every rank from one process."""
    comms = [ShardComm(cfg, r, world, n_reads) for r in range(world)]
    for c in comms:
        for o in comms:
            if o is not c:
                c.set_peer(o)
    return comms


class ShardedCall:
    """One sharded memory-layer forward on one rank, with its buffers kept
    alive so that the three phases can be run separately."""

    def __init__(self, layer: MemoryLayer, comm: ShardComm, params: Dict, h: torch.Tensor, *,
                 train: bool = False, noise_scale: float = 1.0,
                 shuffle_reads: bool = False, rngs=None, gumbel=None, stats: bool = False):
        P = layer.pool
        self.layer, self.comm, self.stats = layer, comm, stats
        h = _cuda_f32(h, "h")
        self.lead = tuple(h.shape[:-1])
        M = int(math.prod(self.lead)) if self.lead else 1
        device = h.device
        if device.index != comm.device:
            raise ValueError(f"h is on {device}, the communicator on cuda:{comm.device}")
        pool = params["pool"]
        values = pool["values"]
        if M > comm.cfg.tokens:
            raise ValueError(f"{M} tokens exceed the communicator's capacity {comm.cfg.tokens}")
        want = shard_rows(P.pool_size, comm.rank, comm.world)
        if values.shape[0] != want:
            raise ValueError(f"rank {comm.rank} holds {want} rows, values has {values.shape[0]}")
        self.cfg = P.config(M, values.dtype, layer.d_model)
        r, g_, o = (params[f"{n}_{layer.layer}"] for n in ("router", "mem_gate", "mem_out"))
        a, self.keep = P._pool_args(pool, M, device, train=train, noise_scale=noise_scale,
                                    shuffle_reads=shuffle_reads, rngs=rngs, gumbel=gumbel, stats=stats)
        self.w = {k: _cuda_f32(v, k) for k, v in (("wr", r["kernel"]), ("br", r["bias"]), ("wg", g_["kernel"]),
                                                  ("bg", g_["bias"]), ("wo", o["kernel"]), ("bo", o["bias"]))}
        self.h = h
        self.y = torch.empty(*self.lead, layer.d_model, dtype=torch.float32, device=device)
        self.mem = torch.empty(*self.lead, P.d_value, dtype=torch.float32, device=device)
        w = self.w
        self.args = L.MemlayerLayerArgs(h=h.data_ptr(), w_router=_ptr(w["wr"]), b_router=_ptr(w["br"]),
                                        w_gate=_ptr(w["wg"]), b_gate=_ptr(w["bg"]), w_out=_ptr(w["wo"]),
                                        b_out=_ptr(w["bo"]), y=self.y.data_ptr(), mem=self.mem.data_ptr(), pool=a)
        nbytes = C.c_size_t()
        L.check(L.lib().memlayer_shard_workspace_size(C.byref(self.cfg), comm.world, 1, C.byref(nbytes)),
                "memlayer_shard_workspace_size")
        self.nbytes = nbytes.value
        self.ws = _workspace(self.nbytes, device)

    def run(self, phases: int = L.PHASE_ALL, stream: Optional[torch.cuda.Stream] = None) -> None:
        s = (stream or torch.cuda.current_stream(self.h.device)).cuda_stream
        L.check(L.lib().memlayer_layer_forward_sharded(C.byref(self.cfg), C.byref(self.args), self.comm.handle,
                                                       phases, self.ws.data_ptr(), self.nbytes, s),
                "memlayer_layer_forward_sharded")

    def check(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        s = (stream or torch.cuda.current_stream(self.h.device)).cuda_stream
        _raise_device_status(self.cfg, self.ws, s)

    def result(self):
        """(y, mem, aux) as MemoryLayer.apply returns them."""
        return self.y, self.mem, self.layer.pool._aux(self.keep, self.lead, self.stats)


class ShardedBackward:
    """The backward of one :class:`ShardedCall` (memlayer_layer_backward_sharded)
    on the same communicator, once per forward and after it.  Like the
    forward, its three phases can be run separately: ROUTE publishes this
    rank's probe rows, GATHER computes this owner's dots for every rank's
    reads of its rows, REDUCE finishes this rank's gradients."""

    def __init__(self, call: ShardedCall, dy: torch.Tensor, *, balance_coef: float = 0.0,
                 route_through_pool: bool = False):
        if balance_coef != 0.0 and not call.stats:
            raise ValueError("balance_coef != 0 needs the forward run with stats=True")
        self.call = call
        M = call.cfg.tokens
        dy = _cuda_f32(dy, "dy").reshape(M, call.layer.d_model)
        self.g, self.ga, self.ws, self.nbytes = call.layer._grad_setup(call.cfg, M, call.h.device, dy, balance_coef,
                                                                       route_through_pool, call.ws)

    def run(self, phases: int = L.PHASE_ALL, stream: Optional[torch.cuda.Stream] = None) -> None:
        c = self.call
        s = (stream or torch.cuda.current_stream(c.h.device)).cuda_stream
        L.check(L.lib().memlayer_layer_backward_sharded(C.byref(c.cfg), C.byref(c.args), C.byref(self.ga),
                                                        c.comm.handle, phases, self.ws.data_ptr(), self.nbytes, s),
                "memlayer_layer_backward_sharded")

    def check(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        s = (stream or torch.cuda.current_stream(self.call.h.device)).cuda_stream
        _raise_device_status(self.call.cfg, self.ws, s)

    def result(self) -> Dict:
        """The gradients of this rank's tokens, keyed as MemoryLayer.backward's."""
        return self.call.layer._grad_result(self.g)


class ShardedMemoryLayer:
    """MemoryLayer whose value table is row-sharded over a communicator's
    ranks.  ``params["pool"]["values"]`` is this rank's local shard
    (:func:`shard_values`)."""

    def __init__(self, layer: MemoryLayer, comm: ShardComm):
        self.layer, self.comm = layer, comm

    @property
    def pool(self) -> MemoryPool:
        return self.layer.pool

    @on_stream
    def apply(self, params, h: torch.Tensor, *, check: bool = False, stream=None, split: bool = True, **kw):
        """``split``: exchange in two token halves, the second half's push
        overlapping the first half's gather (MEMLAYER_PHASE_SPLIT)."""
        call = ShardedCall(self.layer, self.comm, params, h, **kw)
        call.run(L.PHASE_ALL | (L.PHASE_SPLIT if split else 0), stream)
        if check:
            call.check(stream)
        return call.result()

    @on_stream
    def apply_train(self, params, h: torch.Tensor, *, check: bool = False, stream=None, split: bool = False, **kw):
        """The training forward (selection noise and routing statistics on,
        as MemoryLayer.apply_train): returns (y, mem, aux, ctx), ``ctx`` for
        :meth:`backward`."""
        kw.setdefault("train", True)
        kw.setdefault("stats", True)
        call = ShardedCall(self.layer, self.comm, params, h, **kw)
        call.run(L.PHASE_ALL | (L.PHASE_SPLIT if split else 0), stream)
        if check:
            call.check(stream)
        return call.result() + (call,)

    @on_stream
    def backward(self, ctx: ShardedCall, dy: torch.Tensor, *, balance_coef: float = 0.0,
                 route_through_pool: bool = False, check: bool = False, stream=None) -> Dict:
        """MemoryLayer.backward for this rank's tokens; every rank calls it
        for the same forward.  The Dense, sub-key and temperature gradients
        are this rank's share, to be summed over the ranks."""
        b = ShardedBackward(ctx, dy, balance_coef=balance_coef, route_through_pool=route_through_pool)
        b.run(L.PHASE_ALL, stream)
        if check:
            b.check(stream)
        return b.result()


class StagedCall:
    """One row-sharded memory-layer forward whose exchange runs through the
    caller's collectives (memlayer_layer_forward_staged): ROUTE, an
    all-gather of every rank's (slot, weight) entries, GATHER of this rank's
    rows for every rank's tokens, a reduce-scatter of the partial rows, then
    REDUCE (gate and output projection).  :meth:`run` uses NCCL through
    ``torch.distributed``; the phases can also be driven one at a time
    (tests emulate the collectives on one GPU).  Every rank passes the same
    number of tokens."""

    def __init__(self, layer: MemoryLayer, params: Dict, h: torch.Tensor, rank: int, world: int, *,
                 train: bool = False, noise_scale: float = 1.0, shuffle_reads: bool = False, rngs=None,
                 gumbel=None, stats: bool = False):
        P = layer.pool
        self.layer, self.rank, self.world, self.stats = layer, rank, world, stats
        h = _cuda_f32(h, "h")
        self.lead = tuple(h.shape[:-1])
        M = int(math.prod(self.lead)) if self.lead else 1
        device = h.device
        pool = params["pool"]
        values = pool["values"]
        want = shard_rows(P.pool_size, rank, world)
        if values.shape[0] != want:
            raise ValueError(f"rank {rank} holds {want} rows, values has {values.shape[0]}")
        self.cfg = P.config(M, values.dtype, layer.d_model)
        hk = P.heads * P.top_k
        # this rank's slots and weight bits land in its block of the packed
        # [world][2][M*H*k] buffer that one all-gather fills
        self.route = torch.empty(world, 2, M * hk, dtype=torch.int32, device=device)
        self.partials = torch.empty(world, M, P.d_value, dtype=torch.float32, device=device)
        self.mem_in = torch.empty(M, P.d_value, dtype=torch.float32, device=device)
        r, g_, o = (params[f"{n}_{layer.layer}"] for n in ("router", "mem_gate", "mem_out"))
        a, self.keep = P._pool_args(pool, M, device, train=train, noise_scale=noise_scale,
                                    shuffle_reads=shuffle_reads, rngs=rngs, gumbel=gumbel, stats=stats)
        mine = self.route[rank]
        a.slots, a.weights = mine[0].data_ptr(), mine[1].data_ptr()
        self.keep["slots"] = mine[0].view(M, P.heads, P.top_k)
        self.keep["weights"] = mine[1].view(torch.float32).view(M, P.heads, P.top_k)
        self.w = {k: _cuda_f32(v, k) for k, v in (("wr", r["kernel"]), ("br", r["bias"]), ("wg", g_["kernel"]),
                                                  ("bg", g_["bias"]), ("wo", o["kernel"]), ("bo", o["bias"]))}
        self.h = h
        self.y = torch.empty(*self.lead, layer.d_model, dtype=torch.float32, device=device)
        self.mem = torch.empty(*self.lead, P.d_value, dtype=torch.float32, device=device)
        w = self.w
        self.args = L.MemlayerLayerArgs(h=h.data_ptr(), w_router=_ptr(w["wr"]), b_router=_ptr(w["br"]),
                                        w_gate=_ptr(w["wg"]), b_gate=_ptr(w["bg"]), w_out=_ptr(w["wo"]),
                                        b_out=_ptr(w["bo"]), y=self.y.data_ptr(), mem=self.mem.data_ptr(), pool=a)
        self.sargs = L.MemlayerStagedArgs(all_slots=self.route.data_ptr(), all_weights=self.route[0, 1].data_ptr(),
                                          route_stride=2 * M * hk, partials=self.partials.data_ptr(),
                                          mem=self.mem_in.data_ptr(), rank=rank, world=world)
        nbytes = C.c_size_t()
        L.check(L.lib().memlayer_layer_workspace_size(C.byref(self.cfg), C.byref(nbytes)),
                "memlayer_layer_workspace_size")
        self.nbytes = nbytes.value
        self.ws = _workspace(self.nbytes, device)

    def phase(self, ph: int, stream: Optional[torch.cuda.Stream] = None) -> None:
        s = (stream or torch.cuda.current_stream(self.h.device)).cuda_stream
        L.check(L.lib().memlayer_layer_forward_staged(C.byref(self.cfg), C.byref(self.args), C.byref(self.sargs),
                                                      ph, self.ws.data_ptr(), self.nbytes, s),
                "memlayer_layer_forward_staged")

    def run(self, group=None) -> None:
        """All phases with NCCL between them, on the current stream."""
        import torch.distributed as dist
        self.phase(L.PHASE_ROUTE)
        dist.all_gather_into_tensor(self.route.view(-1), self.route[self.rank].view(-1), group=group)
        self.phase(L.PHASE_GATHER)
        dist.reduce_scatter_tensor(self.mem_in.view(-1), self.partials.view(-1), group=group)
        self.phase(L.PHASE_REDUCE)

    def check(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        s = (stream or torch.cuda.current_stream(self.h.device)).cuda_stream
        _raise_device_status(self.cfg, self.ws, s)

    def result(self):
        """(y, mem, aux) as MemoryLayer.apply returns them."""
        return self.y, self.mem, self.layer.pool._aux(self.keep, self.lead, self.stats)
