"""Decode steps of the memory layer as replayable CUDA graphs.

The reference generates token by token with a jitted one-token step
(memory_pool_model/generate.py:23-34 ``Generator._step``: the model in
decode mode on ``tokens[:, None]``), in which every memory layer runs on
the batch's newest position.  ``LayerDecodeStep`` is that memory-layer call
for a fixed batch: the C-ABI call ``memlayer_layer_forward`` (router GEMM,
product-key search, gather, gate, output projection) is built once on
static device buffers, warmed up, and captured into a CUDA graph; each step
copies the new hidden states in and replays the graph, so a decode step
costs one graph launch instead of the call's host work and its kernel
launches.  The captured call is ``memlayer_layer_forward_prepared``: the
sub-key normalisation and the Dense-kernel preparation done by the warm-up
call stay in the workspace, since the weights do not change between decode
steps (``refresh()`` redoes them after a weight update).  Outputs are
bit-identical to ``MemoryLayer.apply`` on the same inputs.

The backbone around the layer (embedding, attention with its KV cache,
feed-forward blocks, logits: model.py:15-127) is not part of this package.
"""

from __future__ import annotations

import ctypes as C
from typing import Any, Dict, Optional, Tuple

import torch

from . import _lib as L
from .memory import MemoryLayer, _cuda_f32, _ptr, _workspace


class LayerDecodeStep:
    """One memory layer's call for ``batch`` new tokens per decode step.

    ``step(h)`` (h [batch, d_model]) returns ``(y, mem, aux)`` like
    ``MemoryLayer.apply(params, h)``; ``y`` / ``mem`` / ``aux`` are views of
    static buffers, overwritten by the next step (clone to keep them).
    ``graph=False`` issues the call directly each step (same results)."""

    def __init__(self, layer: MemoryLayer, params: Dict[str, Any], batch: int, *, graph: bool = True,
                 shuffle_reads: bool = False, device: Optional[torch.device] = None):
        P = layer.pool
        self.layer, self.batch = layer, batch
        device = device or torch.device("cuda", torch.cuda.current_device())
        self.device = device
        if batch < 1:
            raise ValueError("batch must be at least 1")
        r, g_, o = (params[f"{n}_{layer.layer}"] for n in ("router", "mem_gate", "mem_out"))
        values = params["pool"]["values"]
        self.cfg = P.config(batch, values.dtype, layer.d_model)
        self.h = torch.zeros(batch, layer.d_model, dtype=torch.float32, device=device)
        self.y = torch.empty(batch, layer.d_model, dtype=torch.float32, device=device)
        self.mem = torch.empty(batch, P.d_value, dtype=torch.float32, device=device)
        a, self._keep = P._pool_args(params["pool"], batch, device, train=False, noise_scale=1.0,
                                     shuffle_reads=shuffle_reads, rngs=None, gumbel=None, stats=False)
        self._w = {k: _cuda_f32(v, k) for k, v in (("wr", r["kernel"]), ("br", r["bias"]), ("wg", g_["kernel"]),
                                                   ("bg", g_["bias"]), ("wo", o["kernel"]), ("bo", o["bias"]))}
        w = self._w
        self.args = L.MemlayerLayerArgs(h=self.h.data_ptr(), w_router=_ptr(w["wr"]), b_router=_ptr(w["br"]),
                                        w_gate=_ptr(w["wg"]), b_gate=_ptr(w["bg"]), w_out=_ptr(w["wo"]),
                                        b_out=_ptr(w["bo"]), y=self.y.data_ptr(), mem=self.mem.data_ptr(), pool=a)
        nbytes = C.c_size_t()
        L.check(L.lib().memlayer_layer_workspace_size(C.byref(self.cfg), C.byref(nbytes)),
                "memlayer_layer_workspace_size")
        self.nbytes = nbytes.value
        self.ws = _workspace(self.nbytes, device)
        self.graph = None
        s = torch.cuda.Stream(device)
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s):
            self._call(s, prepared=False)     # prepares sub-keys and Dense kernels in the workspace
            self._call(s, prepared=True)      # sets kernel attributes outside the capture
        s.synchronize()
        if graph:
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph, stream=s):
                self._call(s, prepared=True)
        torch.cuda.current_stream(device).wait_stream(s)

    def _call(self, stream: torch.cuda.Stream, prepared: bool = True) -> None:
        lib = L.lib()
        f = lib.memlayer_layer_forward_prepared if prepared else lib.memlayer_layer_forward
        L.check(f(C.byref(self.cfg), C.byref(self.args), self.ws.data_ptr(), self.nbytes, stream.cuda_stream),
                "memlayer_layer_forward")

    def refresh(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Redo the sub-key and Dense-kernel preparation after the layer's
        weights changed in place (the graph keeps reading the same buffers)."""
        s = stream or torch.cuda.current_stream(self.device)
        with torch.cuda.stream(s):
            self._call(s, prepared=False)

    def step(self, h: torch.Tensor, stream: Optional[torch.cuda.Stream] = None
             ) -> Tuple[torch.Tensor, torch.Tensor, Dict[str, torch.Tensor]]:
        if tuple(h.shape) != (self.batch, self.layer.d_model):
            raise ValueError(f"h must be [{self.batch}, {self.layer.d_model}]")
        s = stream or torch.cuda.current_stream(self.device)
        with torch.cuda.stream(s):
            self.h.copy_(h, non_blocking=True)
            if self.graph is not None:
                self.graph.replay()
            else:
                self._call(s)
        P = self.layer.pool
        aux = {"slots": self._keep["slots"].reshape(self.batch, P.heads, P.top_k),
               "weights": self._keep["weights"].reshape(self.batch, P.heads, P.top_k),
               "temperature": self._keep["temperature"].reshape(()),
               "top1_weight": self._keep["top1"].reshape(())}
        return self.y, self.mem, aux

    def status(self) -> int:
        """The device status word of the last step (synchronises)."""
        return L.device_status(self.cfg, self.ws.data_ptr(), torch.cuda.current_stream(self.device).cuda_stream)


def decode_steps_per_second(step: LayerDecodeStep, n: int = 100) -> float:
    """Host-observed decode rate: issue, run and wait for ``n`` steps one at a
    time (each waits for the previous one, as a token-by-token loop does)."""
    import time
    h = torch.randn(step.batch, step.layer.d_model, device=step.device)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(n):
        step.step(h)
        torch.cuda.current_stream(step.device).synchronize()
    return n / (time.perf_counter() - t0)
