"""Host-side mirror of the reference language model and its decoder.

``MemoryPoolLM`` covers ``MemoryPoolLM.__call__`` of
memory_pool_model/model.py:15-127 in inference form (dropout off; routing
statistics through ``MemoryLayer.apply_train``) and ``Generator`` the
token-by-token loop of generate.py:23-65.  Parameters use the reference's
Flax tree (``embed/embedding``, ``pos_embed``, ``ln_attn_i``, ``attn_i``
with ``query`` / ``key`` / ``value`` / ``out``, ``ln_ffn_i``, ``ffn_in_i``,
``ffn_out_i``, ``router_i``, ``mem_gate_i``, ``mem_out_i``, ``pool``,
``ln_final``) as torch CUDA tensors; every step runs in ``libmemlayer.so``
(``memlayer_model_forward``, ``memlayer_model_decode_step``).  A decode step
is captured once as a CUDA graph and replayed for every position.
"""

from __future__ import annotations

import ctypes as C
import dataclasses
import math
import time
from typing import Any, Dict, Tuple

import numpy as np
import torch

from . import _lib as L
from .memory import MemoryPool, _cuda_f32, _raise_device_status, _workspace


@dataclasses.dataclass(frozen=True)
class ModelConfig:
    """The fields of the reference's ModelConfig (config.py:9-59) that the
    forward reads, with its defaults."""

    vocab_size: int = 256
    max_len: int = 128
    d_model: int = 128
    n_layers: int = 2
    n_heads: int = 4
    ffn_mult: int = 1
    dropout: float = 0.0
    use_memory: bool = True
    memory_layers: Tuple[int, ...] = (1,)
    memory_ffn: bool = False
    n_sub_keys: int = 64
    pool_heads: int = 4
    d_key: int = 64
    d_value: int = 128
    top_k: int = 16
    routing_noise: float = 1.0
    init_temperature: float = 10.0
    min_temperature: float = 10.0
    balance_temperature_grad: bool = False
    max_temperature: float = 100.0
    router_query_scale: bool = False

    @property
    def pool_size(self) -> int:
        return self.n_sub_keys ** 2


class MemoryPoolLM:
    """Causal LM: backbone + router + one shared memory pool (model.py:15-127)."""

    def __init__(self, cfg: ModelConfig):
        self.cfg = cfg
        self.pool = MemoryPool(n_sub_keys=cfg.n_sub_keys, heads=cfg.pool_heads, d_key=cfg.d_key,
                               d_value=cfg.d_value, top_k=cfg.top_k, routing_noise=cfg.routing_noise,
                               init_temperature=cfg.init_temperature, min_temperature=cfg.min_temperature,
                               balance_temperature_grad=cfg.balance_temperature_grad,
                               max_temperature=cfg.max_temperature, query_scale=cfg.router_query_scale)

    @property
    def memory_layers(self) -> Tuple[int, ...]:
        return tuple(i for i in self.cfg.memory_layers if i < self.cfg.n_layers) if self.cfg.use_memory else ()

    def config(self, values_dtype=torch.float32) -> L.MemlayerModelConfig:
        c = self.cfg
        mask = 0
        for i in self.memory_layers:
            mask |= 1 << i
        return L.MemlayerModelConfig(vocab_size=c.vocab_size, max_len=c.max_len, d_model=c.d_model,
                                     n_layers=c.n_layers, n_heads=c.n_heads, ffn_mult=c.ffn_mult,
                                     memory_layers=mask, memory_ffn=int(c.memory_ffn),
                                     pool=self.pool.config(0, values_dtype, c.d_model))

    def init(self, seed: int = 0, device="cuda", values_dtype=torch.float32) -> Dict[str, Any]:
        """Parameters with the reference's shapes and initialisers: nn.Embed
        normal(1), pos_embed normal(0.02), lecun-normal Dense kernels with
        zero biases, LayerNorm ones / zeros, the pool as MemoryPool.init."""
        c, P = self.cfg, self.pool
        g = torch.Generator(device="cpu").manual_seed(seed)
        dm, H = c.d_model, c.n_heads
        dh = dm // H

        def t(x):
            return x.to(device)

        def lecun(fan_in, *shape):
            return t(torch.randn(*shape, generator=g) / math.sqrt(fan_in))

        def dense(fi, fo):
            return {"kernel": lecun(fi, fi, fo), "bias": t(torch.zeros(fo))}

        def ln():
            return {"scale": t(torch.ones(dm)), "bias": t(torch.zeros(dm))}

        p: Dict[str, Any] = {"embed": {"embedding": t(torch.randn(c.vocab_size, dm, generator=g))},
                             "pos_embed": t(torch.randn(c.max_len, dm, generator=g) * 0.02)}
        for i in range(c.n_layers):
            p[f"ln_attn_{i}"] = ln()
            p[f"attn_{i}"] = {n: {"kernel": lecun(dm, dm, H, dh), "bias": t(torch.zeros(H, dh))}
                              for n in ("query", "key", "value")}
            p[f"attn_{i}"]["out"] = {"kernel": lecun(dm, H, dh, dm), "bias": t(torch.zeros(dm))}
            p[f"ln_ffn_{i}"] = ln()
            if i not in self.memory_layers or c.memory_ffn:
                p[f"ffn_in_{i}"] = dense(dm, dm * c.ffn_mult)
                p[f"ffn_out_{i}"] = dense(dm * c.ffn_mult, dm)
            if i in self.memory_layers:
                p[f"router_{i}"] = dense(dm, P.heads * P.d_key)
                p[f"mem_gate_{i}"] = dense(dm, P.d_value)
                p[f"mem_out_{i}"] = dense(P.d_value, dm)
        if self.memory_layers:
            p["pool"] = P.init(seed, device, values_dtype)["params"]
        p["ln_final"] = ln()
        return p

    def prepare(self, params) -> "PreparedModel":
        """The C ABI's view of ``params`` (attention kernels reshaped and the
        query / key / value kernels concatenated once); reuse it across calls
        while the parameters are unchanged."""
        return PreparedModel(self, params)

    def apply(self, params, tokens: torch.Tensor, *, check: bool = False, stream=None):
        """MemoryPoolLM.__call__(tokens) with train=False: (logits [B, T, V], aux).
        Routing statistics are not produced here (aux is empty)."""
        prep = params if isinstance(params, PreparedModel) else self.prepare(params)
        return prep.forward(tokens, check=check, stream=stream), {}


class PreparedModel:
    """Parameters of one MemoryPoolLM laid out for the C ABI."""

    def __init__(self, model: MemoryPoolLM, params):
        self.model = model
        c = model.cfg
        dm = c.d_model
        f = lambda x, n: _cuda_f32(x, n)  # noqa: E731
        keep = []

        def ptr(x):
            if x is None:
                return None
            keep.append(x)
            return x.data_ptr()

        self.embedding = f(params["embed"]["embedding"], "embedding")
        self.pos_embed = f(params["pos_embed"], "pos_embed")
        blocks = (L.MemlayerBlockParams * max(1, c.n_layers))()
        for i in range(c.n_layers):
            a = params[f"attn_{i}"]
            w_qkv = torch.cat([f(a[n]["kernel"], n).reshape(dm, dm) for n in ("query", "key", "value")], 1)
            b_qkv = torch.cat([f(a[n]["bias"], n).reshape(dm) for n in ("query", "key", "value")])
            b = blocks[i]
            b.ln_attn_scale, b.ln_attn_bias = (ptr(f(params[f"ln_attn_{i}"][k], k)) for k in ("scale", "bias"))
            b.w_qkv, b.b_qkv = ptr(w_qkv.contiguous()), ptr(b_qkv.contiguous())
            b.w_attn_out = ptr(f(a["out"]["kernel"], "out").reshape(dm, dm))
            b.b_attn_out = ptr(f(a["out"]["bias"], "out bias"))
            b.ln_ffn_scale, b.ln_ffn_bias = (ptr(f(params[f"ln_ffn_{i}"][k], k)) for k in ("scale", "bias"))
            if f"ffn_in_{i}" in params:
                b.w_ffn_in, b.b_ffn_in = (ptr(f(params[f"ffn_in_{i}"][k], k)) for k in ("kernel", "bias"))
                b.w_ffn_out, b.b_ffn_out = (ptr(f(params[f"ffn_out_{i}"][k], k)) for k in ("kernel", "bias"))
            if i in model.memory_layers:
                b.w_router, b.b_router = (ptr(f(params[f"router_{i}"][k], k)) for k in ("kernel", "bias"))
                b.w_gate, b.b_gate = (ptr(f(params[f"mem_gate_{i}"][k], k)) for k in ("kernel", "bias"))
                b.w_out, b.b_out = (ptr(f(params[f"mem_out_{i}"][k], k)) for k in ("kernel", "bias"))
        self.values_dtype = torch.float32
        mp = L.MemlayerModelParams(embedding=self.embedding.data_ptr(), pos_embed=self.pos_embed.data_ptr(),
                                   layers=C.cast(blocks, C.POINTER(L.MemlayerBlockParams)),
                                   ln_final_scale=ptr(f(params["ln_final"]["scale"], "ln_final")),
                                   ln_final_bias=ptr(f(params["ln_final"]["bias"], "ln_final")))
        if model.memory_layers:
            pool = params["pool"]
            values = pool["values"]
            if not values.is_cuda or not values.is_contiguous():
                raise TypeError("pool values must be a contiguous CUDA tensor")
            self.values_dtype = values.dtype
            keep.append(values)
            mp.sub_keys = ptr(f(pool["sub_keys"], "sub_keys"))
            mp.log_temperature = ptr(f(torch.as_tensor(pool["log_temperature"], device=values.device).reshape(1),
                                       "log_temperature"))
            mp.values = values.data_ptr()
        self._keep, self._blocks, self.params = keep, blocks, mp
        self.cfg = model.config(self.values_dtype)
        self.device = self.embedding.device

    def workspace_bytes(self, rows: int) -> int:
        nb = C.c_size_t()
        L.check(L.lib().memlayer_model_workspace_size(C.byref(self.cfg), rows, C.byref(nb)),
                "memlayer_model_workspace_size")
        return nb.value

    def forward(self, tokens: torch.Tensor, *, check: bool = False, stream=None) -> torch.Tensor:
        if tokens.dim() != 2:
            raise ValueError("tokens must be [batch, seq]")
        B, T = tokens.shape
        tok = tokens.to(self.device, torch.int32).contiguous()
        logits = torch.empty(B, T, self.model.cfg.vocab_size, dtype=torch.float32, device=self.device)
        nb = self.workspace_bytes(B * T)
        ws = _workspace(nb, self.device)
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        L.check(L.lib().memlayer_model_forward(C.byref(self.cfg), C.byref(self.params), tok.data_ptr(), B, T,
                                               logits.data_ptr(), ws.data_ptr(), nb, s), "memlayer_model_forward")
        if check:
            _raise_device_status(self.cfg.pool, ws, s)
        return logits


class Generator:
    """Token-by-token generation with a key / value cache (generate.py:23-65).
    The decode step is captured once as a CUDA graph (static token, position
    and logits buffers; the position is read on the GPU) and replayed for
    every position; ``graph=False`` issues it eagerly."""

    def __init__(self, model: MemoryPoolLM, params, batch_size: int = 1, graph: bool = True):
        self.model, self.batch_size = model, batch_size
        self.prep = params if isinstance(params, PreparedModel) else model.prepare(params)
        dev = self.prep.device
        c = model.cfg
        nb = C.c_size_t()
        L.check(L.lib().memlayer_model_cache_size(C.byref(self.prep.cfg), batch_size, C.byref(nb)),
                "memlayer_model_cache_size")
        self.cache = _workspace(nb.value, dev)
        self.ws_bytes = self.prep.workspace_bytes(batch_size)
        self.ws = _workspace(self.ws_bytes, dev)
        self.tok = torch.zeros(batch_size, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.logits = torch.empty(batch_size, c.vocab_size, dtype=torch.float32, device=dev)
        self.stream = torch.cuda.Stream(dev)
        self.graph = None
        if graph:
            self._step_eager()                     # warm-up outside the capture
            self.stream.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=self.stream):
                self._step_eager()

    def _step_eager(self):
        L.check(L.lib().memlayer_model_decode_step(C.byref(self.prep.cfg), C.byref(self.prep.params),
                                                   self.tok.data_ptr(), self.batch_size, self.pos.data_ptr(),
                                                   self.cache.data_ptr(), self.logits.data_ptr(), self.ws.data_ptr(),
                                                   self.ws_bytes, torch.cuda.current_stream().cuda_stream),
                "memlayer_model_decode_step")

    def step(self, tokens: torch.Tensor, pos: int) -> torch.Tensor:
        """logits [B, V] of tokens [B] at position pos (generate.py:31-34)."""
        with torch.cuda.stream(self.stream):
            self.tok.copy_(tokens.to(self.tok.device, torch.int32), non_blocking=True)
            self.pos.fill_(int(pos))
            if self.graph is not None:
                self.graph.replay()
            else:
                self._step_eager()
        return self.logits

    def status(self) -> int:
        return L.device_status(self.prep.cfg.pool, self.ws.data_ptr(), self.stream.cuda_stream)

    def generate(self, prompt, n_new: int, temperature: float = 0.0, seed: int = 0) -> Dict[str, object]:
        """prompt [B, P] int tokens; greedy when temperature == 0, else
        sampled from softmax(logits / temperature) (torch's generator, not
        JAX's).  Returns tokens, every step's logits and per-step wall times
        (generate.py:36-63)."""
        prompt = np.asarray(prompt, np.int32)
        B, P = prompt.shape
        if B != self.batch_size:
            raise ValueError(f"prompt batch {B} != generator batch {self.batch_size}")
        if P + n_new > self.model.cfg.max_len:
            raise ValueError("prompt + n_new exceeds max_len")
        dev = self.prep.device
        g = torch.Generator(device=dev).manual_seed(seed)
        tok = torch.as_tensor(prompt[:, 0], device=dev)
        out, logits_all, times = [], [], []
        for pos in range(P + n_new - 1):
            t0 = time.perf_counter()
            logits = self.step(tok, pos)
            with torch.cuda.stream(self.stream):
                if pos + 1 < P:
                    nxt = torch.as_tensor(prompt[:, pos + 1], device=dev)
                elif temperature > 0:
                    nxt = torch.multinomial(torch.softmax(logits / temperature, -1), 1, generator=g)[:, 0]
                else:
                    nxt = torch.argmax(logits, -1)
                lg = logits.clone()
            self.stream.synchronize()
            times.append(time.perf_counter() - t0)
            logits_all.append(lg)
            if pos + 1 >= P:
                out.append(nxt.to(torch.int32))
            tok = nxt
        code = self.status()
        if code:
            raise L.DeviceError(f"device status {code}: {L.DEVICE_ERRORS.get(code, 'unknown')}")
        return {"tokens": torch.stack(out, 1).cpu().numpy() if out else np.zeros((B, 0), np.int32),
                "logits": torch.stack(logits_all, 1).cpu().numpy(), "step_seconds": np.array(times)}
