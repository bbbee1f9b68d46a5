"""Host-side mirror of the reference memory layer over the CUDA C ABI.

``MemoryPool`` keeps the field names, defaults, parameter names, call
signature, aux dictionary and assertion behaviour of the reference's Flax
module (memory_pool_model/memory.py:64-227); ``MemoryLayer`` covers the
router / gate / output projections around it (model.py:108-120).  Arrays are
torch tensors on a CUDA device; every step runs in ``libmemlayer.so``.
There is no CPU path: a tensor on another device raises.
"""

from __future__ import annotations

import ctypes as C
import dataclasses
import functools
import math
from typing import Any, Dict, Optional, Tuple

import torch

from . import _lib as L

_DTYPES = {torch.float32: L.F32, torch.float16: L.F16, torch.bfloat16: L.BF16}


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _cuda_f32(t: torch.Tensor, name: str) -> torch.Tensor:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor (no CPU path)")
    return t.to(torch.float32).contiguous()


def _raise_device_status(cfg, ws: torch.Tensor, stream_ptr: int) -> None:
    code = L.device_status(cfg, ws.data_ptr(), stream_ptr)
    if code:
        raise L.DeviceError(f"device status {code}: {L.DEVICE_ERRORS.get(code, 'unknown')}")


def _workspace(nbytes: int, device) -> torch.Tensor:
    # torch's caching allocator hands out 512-byte aligned blocks
    return torch.empty(max(nbytes, 256), dtype=torch.uint8, device=device)


def on_stream(fn):
    """Runs ``fn`` with its ``stream`` keyword argument as the current CUDA
    stream.  The workspaces, converted inputs and outputs that ``fn``
    allocates then belong to the stream its kernels run on: the caching
    allocator reuses a block freed when ``fn`` returns only in that stream's
    order, never while the kernels still read it."""
    @functools.wraps(fn)
    def wrapped(*args, stream: Optional[torch.cuda.Stream] = None, **kw):
        if stream is None:
            return fn(*args, stream=None, **kw)
        with torch.cuda.stream(stream):
            return fn(*args, stream=stream, **kw)
    return wrapped


@dataclasses.dataclass
class MemoryPool:
    """A pool of ``n_sub_keys ** 2`` value vectors read through product keys.

    Fields match memory.py:72-97.  ``apply(variables, queries, ...)`` takes
    ``variables = {"params": {"sub_keys", "values", "log_temperature"}}``
    (the reference's parameter names and shapes) and returns
    ``(out [..., d_value], aux)``.
    """

    n_sub_keys: int
    heads: int
    d_key: int
    d_value: int
    top_k: int
    routing_noise: float = 1.0
    init_temperature: float = 10.0
    min_temperature: float = 10.0
    balance_temperature_grad: bool = False
    max_temperature: float = 100.0
    query_scale: bool = False
    host_pool: str = ""

    def __post_init__(self):
        # memory.py:95-96
        assert self.d_key % 2 == 0, "d_key must be even (split into two halves)"
        assert self.top_k <= self.n_sub_keys

    @property
    def pool_size(self) -> int:
        return self.n_sub_keys ** 2

    # -- parameters (memory.py:94-113) --
    def init(self, seed: int = 0, device="cuda", values_dtype=torch.float32,
             values_std: Optional[float] = None) -> Dict[str, Dict[str, torch.Tensor]]:
        """Parameters with the reference's initialisers: unit-sphere sub_keys,
        N(0, d_value^-0.5) values, log(init_temperature)."""
        g = torch.Generator(device="cpu").manual_seed(seed)
        half = self.d_key // 2
        sk = torch.randn(self.heads, 2, self.n_sub_keys, half, generator=g)
        sk = sk * torch.rsqrt((sk * sk).sum(-1, keepdim=True) + 1e-6)
        std = self.d_value ** -0.5 if values_std is None else values_std
        values = (torch.randn(self.pool_size, self.d_value, generator=g) * std).to(values_dtype)
        return {"params": {
            "sub_keys": sk.to(device),
            "values": values.to(device),
            "log_temperature": torch.tensor(math.log(self.init_temperature), dtype=torch.float32, device=device),
        }}

    def config(self, tokens: int, values_dtype: torch.dtype, d_model: int = 0) -> L.MemlayerConfig:
        if values_dtype not in _DTYPES:
            raise TypeError(f"values dtype {values_dtype} is not float32/float16/bfloat16")
        return L.MemlayerConfig(
            tokens=tokens, heads=self.heads, n_sub_keys=self.n_sub_keys, d_key=self.d_key, d_value=self.d_value,
            top_k=self.top_k, d_model=d_model, values_dtype=_DTYPES[values_dtype],
            routing_noise=self.routing_noise, min_temperature=self.min_temperature,
            max_temperature=self.max_temperature, query_scale=int(self.query_scale),
            balance_temperature_grad=int(self.balance_temperature_grad))

    def _noise(self, shape, train: bool, noise_scale: float, rngs, gumbel, device) -> Optional[torch.Tensor]:
        if not (train and self.routing_noise > 0 and noise_scale != 0):
            return None
        if gumbel is None:
            # the reference draws from the "routing" RNG stream (memory.py:156)
            seed = 0 if rngs is None else int(rngs.get("routing", 0)) if isinstance(rngs, dict) else int(rngs)
            gen = torch.Generator(device=device).manual_seed(seed)
            u = torch.rand(shape, generator=gen, device=device).clamp_(min=torch.finfo(torch.float32).tiny)
            gumbel = -torch.log(-torch.log(u))
        return _cuda_f32(gumbel, "gumbel")

    def _values(self, p) -> torch.Tensor:
        """The value table: a CUDA tensor, or with ``host_pool`` the named
        host table's page-locked rows (memory.py:90-92, 180-183)."""
        if self.host_pool:
            from .host_table import get
            return get(self.host_pool).values
        values = p["values"]
        if not values.is_cuda:
            raise TypeError("values must be a CUDA tensor (no CPU path)")
        return values.contiguous()

    def _pool_args(self, params, M, device, *, train, noise_scale, shuffle_reads, rngs, gumbel, stats):
        p = params["params"] if "params" in params else params
        sub_keys = _cuda_f32(p["sub_keys"], "sub_keys")
        values = self._values(p)
        log_t = _cuda_f32(torch.as_tensor(p["log_temperature"], device=device).reshape(1), "log_temperature")
        H, k, n = self.heads, self.top_k, self.n_sub_keys
        keep = dict(sub_keys=sub_keys, values=values, log_t=log_t)
        keep["gumbel"] = self._noise((M, H, 2, n), train, noise_scale, rngs, gumbel, device)
        keep["slots"] = torch.empty(M, H, k, dtype=torch.int32, device=device)
        keep["weights"] = torch.empty(M, H, k, dtype=torch.float32, device=device)
        keep["temperature"] = torch.empty(1, dtype=torch.float32, device=device)
        keep["top1"] = torch.empty(1, dtype=torch.float32, device=device)
        if stats:
            keep["queries_unit"] = torch.empty(M, H, 2, self.d_key // 2, dtype=torch.float32, device=device)
            keep["subkey_counts"] = torch.empty(H, 2, n, dtype=torch.float32, device=device)
            keep["slot_counts"] = torch.empty(self.pool_size, dtype=torch.float32, device=device)
            keep["balance_loss"] = torch.empty(1, dtype=torch.float32, device=device)
        a = L.MemlayerPoolArgs(
            sub_keys=_ptr(sub_keys), log_temperature=_ptr(log_t), values=_ptr(values),
            gumbel=_ptr(keep["gumbel"]), noise_scale=float(noise_scale), train=int(bool(train)),
            shuffle_reads=int(bool(shuffle_reads)), slots=_ptr(keep["slots"]), weights=_ptr(keep["weights"]),
            queries_unit=_ptr(keep.get("queries_unit")), subkey_counts=_ptr(keep.get("subkey_counts")),
            slot_counts=_ptr(keep.get("slot_counts")), balance_loss=_ptr(keep.get("balance_loss")),
            top1_weight=_ptr(keep["top1"]), temperature=_ptr(keep["temperature"]))
        return a, keep

    def _aux(self, keep, lead, stats) -> Dict[str, Any]:
        H, k = self.heads, self.top_k
        aux = {
            "slots": keep["slots"].reshape(*lead, H, k),
            "weights": keep["weights"].reshape(*lead, H, k),
            "temperature": keep["temperature"].reshape(()),
            "top1_weight": keep["top1"].reshape(()),
        }
        if stats:
            aux.update(balance_loss=keep["balance_loss"].reshape(()), subkey_counts=keep["subkey_counts"],
                       slot_counts=keep["slot_counts"], queries=keep["queries_unit"])
        return aux

    @on_stream
    def apply(self, variables, queries: torch.Tensor, *, train: bool = False, sparse_grad: bool = False,
              noise_scale: float = 1.0, shuffle_reads: bool = False, rngs=None,
              gumbel: Optional[torch.Tensor] = None, stats: bool = True,
              stream: Optional[torch.cuda.Stream] = None, check: bool = False) -> Tuple[torch.Tensor, Dict[str, Any]]:
        """MemoryPool.__call__ (memory.py:119-227).  ``gumbel`` optionally
        supplies the standard Gumbel sample used when ``train`` (else one is
        drawn from ``rngs["routing"]``); ``stats=False`` skips the routing
        statistics that only training consumes."""
        del sparse_grad  # affects differentiation only
        queries = _cuda_f32(queries, "queries")
        lead = tuple(queries.shape[:-2])
        if tuple(queries.shape[-2:]) != (self.heads, self.d_key):
            raise ValueError(f"queries must end in [heads={self.heads}, d_key={self.d_key}]")
        M = int(math.prod(lead)) if lead else 1
        device = queries.device
        p = variables["params"] if "params" in variables else variables
        cfg = self.config(M, self._values(p).dtype)
        a, keep = self._pool_args(variables, M, device, train=train, noise_scale=noise_scale,
                                  shuffle_reads=shuffle_reads, rngs=rngs, gumbel=gumbel, stats=stats)
        out = torch.empty(*lead, self.d_value, dtype=torch.float32, device=device)
        a.queries = queries.data_ptr()
        a.out = out.data_ptr()
        nbytes = C.c_size_t()
        lib = L.lib()
        # host_pool: the GPU fetches each distinct row from host memory once per call
        size_fn, fwd_fn = ((lib.memlayer_host_table_workspace_size, lib.memlayer_pool_forward_host_table)
                           if self.host_pool else (lib.memlayer_pool_workspace_size, lib.memlayer_pool_forward))
        L.check(size_fn(C.byref(cfg), C.byref(nbytes)), "workspace size")
        ws = _workspace(nbytes.value, device)
        s = (stream or torch.cuda.current_stream(device)).cuda_stream
        L.check(fwd_fn(C.byref(cfg), C.byref(a), ws.data_ptr(), nbytes.value, s), "pool forward")
        if check:
            _raise_device_status(cfg, ws, s)
        return out, self._aux(keep, lead, stats)


@dataclasses.dataclass
class MemoryLayer:
    """The memory-layer block of MemoryPoolLM (model.py:108-120) for one
    layer index i: router_i Dense -> MemoryPool -> silu(mem_gate_i Dense)
    gate -> mem_out_i Dense.  Parameter names follow the reference's Flax
    tree: ``router_i``, ``mem_gate_i``, ``mem_out_i`` with ``kernel`` /
    ``bias`` leaves, and ``pool`` with the MemoryPool parameters."""

    pool: MemoryPool
    d_model: int
    layer: int = 1

    def __post_init__(self):
        if self.pool.host_pool:
            # the fused block reads the table from HBM; a host table is read
            # through MemoryPool.apply (memlayer_pool_forward_host_table)
            raise NotImplementedError("MemoryLayer needs the value table in device memory; use MemoryPool.apply "
                                      "for a host_pool table")

    def init(self, seed: int = 0, device="cuda", values_dtype=torch.float32) -> Dict[str, Any]:
        g = torch.Generator(device="cpu").manual_seed(seed + 1)
        P = self.pool

        def dense(fan_in, fan_out):  # flax Dense default: lecun_normal kernel, zero bias
            return {"kernel": (torch.randn(fan_in, fan_out, generator=g) / math.sqrt(fan_in)).to(device),
                    "bias": torch.zeros(fan_out, device=device)}
        return {
            f"router_{self.layer}": dense(self.d_model, P.heads * P.d_key),
            f"mem_gate_{self.layer}": dense(self.d_model, P.d_value),
            f"mem_out_{self.layer}": dense(P.d_value, self.d_model),
            "pool": P.init(seed, device, values_dtype)["params"],
        }

    @on_stream
    def apply_host(self, params, h_host: torch.Tensor, *, chunks: int = 4, device="cuda",
                   shuffle_reads: bool = False, stream: Optional[torch.cuda.Stream] = None,
                   check: bool = False):
        """Inference forward with the hidden state and the output in host
        memory (memlayer_layer_forward_host): the host-to-device copy, the
        layer and the device-to-host copy overlap chunk by chunk.  Returns
        (y_host [..., d_model] pinned, aux on the device)."""
        P = self.pool
        if h_host.is_cuda or h_host.dtype != torch.float32:
            raise TypeError("h_host must be a float32 host tensor")
        h_host = h_host.contiguous()
        if not h_host.is_pinned():
            h_host = h_host.pin_memory()
        lead = tuple(h_host.shape[:-1])
        M = int(math.prod(lead)) if lead else 1
        device = torch.device(device)
        r, g_, o = (params[f"{n}_{self.layer}"] for n in ("router", "mem_gate", "mem_out"))
        cfg = P.config(M, params["pool"]["values"].dtype, self.d_model)
        a, keep = P._pool_args(params["pool"], M, device, train=False, noise_scale=1.0,
                               shuffle_reads=shuffle_reads, rngs=None, gumbel=None, stats=False)
        a.top1_weight = None                              # a per-call mean: not produced chunk by chunk
        w = {k: _cuda_f32(v, k) for k, v in (("wr", r["kernel"]), ("br", r["bias"]), ("wg", g_["kernel"]),
                                             ("bg", g_["bias"]), ("wo", o["kernel"]), ("bo", o["bias"]))}
        y = torch.empty(*lead, self.d_model, dtype=torch.float32).pin_memory()
        la = L.MemlayerLayerArgs(h=h_host.data_ptr(), w_router=_ptr(w["wr"]), b_router=_ptr(w["br"]),
                                 w_gate=_ptr(w["wg"]), b_gate=_ptr(w["bg"]), w_out=_ptr(w["wo"]),
                                 b_out=_ptr(w["bo"]), y=y.data_ptr(), mem=None, pool=a)
        nbytes = C.c_size_t()
        L.check(L.lib().memlayer_layer_host_workspace_size(C.byref(cfg), chunks, C.byref(nbytes)),
                "memlayer_layer_host_workspace_size")
        ws = _workspace(nbytes.value, device)
        s = (stream or torch.cuda.current_stream(device)).cuda_stream
        L.check(L.lib().memlayer_layer_forward_host(C.byref(cfg), C.byref(la), chunks, ws.data_ptr(), nbytes.value,
                                                    s), "memlayer_layer_forward_host")
        if check:
            _raise_device_status(cfg, ws, s)
        torch.cuda.current_stream(device).synchronize() if stream is None else stream.synchronize()
        aux = {"slots": keep["slots"].reshape(*lead, P.heads, P.top_k),
               "weights": keep["weights"].reshape(*lead, P.heads, P.top_k),
               "temperature": keep["temperature"].reshape(())}
        return y, aux

    def apply_train(self, params, h: torch.Tensor, *, train: bool = True, noise_scale: float = 1.0,
                    shuffle_reads: bool = False, rngs=None, gumbel=None,
                    stream: Optional[torch.cuda.Stream] = None, check: bool = False):
        """The training forward (routing statistics on) keeping what
        ``backward`` needs: returns (y, mem, aux, ctx)."""
        y, mem, aux, ctx = self._forward(params, h, train=train, noise_scale=noise_scale,
                                         shuffle_reads=shuffle_reads, rngs=rngs, gumbel=gumbel, stats=True,
                                         stream=stream, check=check)
        return y, mem, aux, ctx

    @on_stream
    def backward(self, ctx: Dict[str, Any], dy: torch.Tensor, *, balance_coef: float = 0.0,
                 route_through_pool: bool = False, stream: Optional[torch.cuda.Stream] = None,
                 check: bool = False) -> Dict[str, torch.Tensor]:
        """Gradients of sum(dy * y) + balance_coef * balance_loss for the
        forward of ``ctx`` (memlayer_layer_backward): the reference's
        parameter names (``router_i`` / ``mem_gate_i`` / ``mem_out_i`` kernel
        and bias, ``pool`` sub_keys and log_temperature), ``h``, and
        ``probe`` = d loss / d read output, the row update's input.  The
        forward's read output kept in ``ctx`` is read, not re-gathered; every
        GEMM runs on the library's tensor-core kernels in the call's own
        workspace, so backward calls may overlap."""
        dev = ctx["device"]
        dy = _cuda_f32(dy, "dy").reshape(ctx["M"], self.d_model)
        g, ga, ws, nb = self._grad_setup(ctx["cfg"], ctx["M"], dev, dy, balance_coef, route_through_pool, ctx["ws"])
        s = (stream or torch.cuda.current_stream(dev)).cuda_stream
        L.check(L.lib().memlayer_layer_backward(C.byref(ctx["cfg"]), C.byref(ctx["la"]), C.byref(ga), ws.data_ptr(),
                                                nb, s), "memlayer_layer_backward")
        if check:
            _raise_device_status(ctx["cfg"], ws, s)
        return self._grad_result(g)

    def _grad_setup(self, cfg, M: int, dev, dy: torch.Tensor, balance_coef: float, route_through_pool: bool,
                    forward_ws: torch.Tensor):
        """Gradient outputs, their memlayer_layer_grads and the backward workspace."""
        P = self.pool
        dm, d = self.d_model, P.d_value
        g = {"h": torch.empty(M, dm, device=dev), "w_router": torch.empty(dm, P.heads * P.d_key, device=dev),
             "b_router": torch.empty(P.heads * P.d_key, device=dev),
             "sub_keys": torch.empty(P.heads, 2, P.n_sub_keys, P.d_key // 2, device=dev),
             "log_temperature": torch.empty(1, device=dev), "w_gate": torch.empty(dm, d, device=dev),
             "b_gate": torch.empty(d, device=dev), "w_out": torch.empty(d, dm, device=dev),
             "b_out": torch.empty(dm, device=dev), "probe": torch.empty(M, d, device=dev), "dy": dy}
        ga = L.MemlayerLayerGrads(dy=dy.data_ptr(), balance_coef=float(balance_coef),
                                  route_through_pool=int(bool(route_through_pool)),
                                  forward_workspace=forward_ws.data_ptr(), dh=g["h"].data_ptr(),
                                  dw_router=g["w_router"].data_ptr(), db_router=g["b_router"].data_ptr(),
                                  dsub_keys=g["sub_keys"].data_ptr(), dlog_temperature=g["log_temperature"].data_ptr(),
                                  dw_gate=g["w_gate"].data_ptr(), db_gate=g["b_gate"].data_ptr(),
                                  dw_out=g["w_out"].data_ptr(), db_out=g["b_out"].data_ptr(),
                                  probe=g["probe"].data_ptr())
        nb = C.c_size_t()
        L.check(L.lib().memlayer_layer_backward_workspace_size(C.byref(cfg), int(balance_coef != 0.0), C.byref(nb)),
                "memlayer_layer_backward_workspace_size")
        return g, ga, _workspace(nb.value, dev), nb.value

    def _grad_result(self, g) -> Dict[str, Any]:
        i = self.layer
        return {"h": g["h"], f"router_{i}": {"kernel": g["w_router"], "bias": g["b_router"]},
                f"mem_gate_{i}": {"kernel": g["w_gate"], "bias": g["b_gate"]},
                f"mem_out_{i}": {"kernel": g["w_out"], "bias": g["b_out"]},
                "pool": {"sub_keys": g["sub_keys"], "log_temperature": g["log_temperature"].reshape(())},
                "probe": g["probe"]}

    def apply(self, params, h: torch.Tensor, *, train: bool = False, noise_scale: float = 1.0,
              shuffle_reads: bool = False, rngs=None, gumbel=None, stats: bool = False,
              stream: Optional[torch.cuda.Stream] = None, check: bool = False):
        """Returns (y [..., d_model], mem [..., d_value], aux); y is the term
        model.py:119 adds into the layer's update."""
        y, mem, aux, _ = self._forward(params, h, train=train, noise_scale=noise_scale, shuffle_reads=shuffle_reads,
                                       rngs=rngs, gumbel=gumbel, stats=stats, stream=stream, check=check)
        return y, mem, aux

    @on_stream
    def _forward(self, params, h, *, train, noise_scale, shuffle_reads, rngs, gumbel, stats, stream, check):
        P = self.pool
        h = _cuda_f32(h, "h")
        lead = tuple(h.shape[:-1])
        M = int(math.prod(lead)) if lead else 1
        device = h.device
        r, g_, o = (params[f"{n}_{self.layer}"] for n in ("router", "mem_gate", "mem_out"))
        cfg = P.config(M, params["pool"]["values"].dtype, self.d_model)
        a, keep = P._pool_args(params["pool"], M, device, train=train, noise_scale=noise_scale,
                               shuffle_reads=shuffle_reads, rngs=rngs, gumbel=gumbel, stats=stats)
        w = {k: _cuda_f32(v, k) for k, v in (("wr", r["kernel"]), ("br", r["bias"]), ("wg", g_["kernel"]),
                                             ("bg", g_["bias"]), ("wo", o["kernel"]), ("bo", o["bias"]))}
        y = torch.empty(*lead, self.d_model, dtype=torch.float32, device=device)
        mem = torch.empty(*lead, P.d_value, dtype=torch.float32, device=device)
        la = L.MemlayerLayerArgs(h=h.data_ptr(), w_router=_ptr(w["wr"]), b_router=_ptr(w["br"]),
                                 w_gate=_ptr(w["wg"]), b_gate=_ptr(w["bg"]), w_out=_ptr(w["wo"]),
                                 b_out=_ptr(w["bo"]), y=y.data_ptr(), mem=mem.data_ptr(), pool=a)
        nbytes = C.c_size_t()
        L.check(L.lib().memlayer_layer_workspace_size(C.byref(cfg), C.byref(nbytes)),
                "memlayer_layer_workspace_size")
        ws = _workspace(nbytes.value, device)
        s = (stream or torch.cuda.current_stream(device)).cuda_stream
        L.check(L.lib().memlayer_layer_forward(C.byref(cfg), C.byref(la), ws.data_ptr(), nbytes.value, s),
                "memlayer_layer_forward")
        if check:
            _raise_device_status(cfg, ws, s)
        ctx = {"cfg": cfg, "la": la, "ws": ws, "keep": keep, "w": w, "h": h, "y": y, "mem": mem, "M": M,
               "device": device}
        return y, mem, P._aux(keep, lead, stats), ctx
