"""CPU oracle for the backbone around the memory layer (TEST INFRASTRUCTURE ONLY).

A float32 numpy restatement of the reference's language model and its
decoding loop:

* ``memory_pool_model/model.py:15-127``  ``MemoryPoolLM.__call__``: token and
  position embeddings, per layer LayerNorm -> multi-head causal attention ->
  residual, LayerNorm -> feed-forward (GELU) or the memory layer -> residual,
  final LayerNorm and tied logits (``embed.attend``);
* ``memory_pool_model/generate.py:23-65`` ``Generator``: one token per step
  with a key / value cache, greedy or sampled continuation.

The flax.linen layers the reference builds on are restated from their
published definitions (flax >= 0.8.5, requirements.txt:2):

* ``nn.LayerNorm``: epsilon 1e-6, "fast" variance E[x^2] - E[x]^2 clamped at
  0, y = (x - mean) * (rsqrt(var + eps) * scale) + bias;
* ``nn.MultiHeadDotProductAttention``: query / key / value DenseGeneral to
  [heads, d_model / heads] with bias, query scaled by 1 / sqrt(head_dim)
  before the dot product, masked scores set to the float32 minimum, softmax
  in float32, output DenseGeneral over (heads, head_dim) with bias; in decode
  mode the new key / value are written at the cache index and the query
  attends to cache positions <= index;
* ``nn.gelu``: the tanh approximation 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)));
* ``nn.Embed.attend``: x @ embedding^T.

Only tests/, __graft_entry__ and bench.py's CPU legs import this file.
Parity: the memory layer inside reuses ``memlayer_ref.layer_forward`` (pinned
by the golden fixtures); the backbone restatement is pinned by the reference's
own property test that decoding with the cache reproduces the full forward
(tests/test_memory_pool.py:486-502), restated in tests/test_backbone_oracle.py.
The flax layer definitions themselves are not run here (no JAX / Flax):
parity of the backbone with flax's own code is unpinned.
"""

from __future__ import annotations

import dataclasses
from typing import Dict, Optional, Tuple

import numpy as np

from . import memlayer_ref as ml

F32 = np.float32


@dataclasses.dataclass(frozen=True)
class ModelCfg:
    """The ModelConfig fields of config.py:9-55 that the forward reads."""

    vocab_size: int
    max_len: int
    d_model: int
    n_layers: int
    n_heads: int
    ffn_mult: int
    memory_layers: Tuple[int, ...]
    pool: ml.PoolConfig
    memory_ffn: bool = False


def layer_norm(x, scale, bias, eps=1e-6):
    """flax.linen.LayerNorm (model.py:87,96,124) with its fast variance."""
    x = np.asarray(x, F32)
    mean = np.mean(x, axis=-1, keepdims=True, dtype=F32)
    mean2 = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    var = np.maximum(F32(0), mean2 - mean * mean)
    mul = (F32(1) / np.sqrt(var + F32(eps))).astype(F32) * np.asarray(scale, F32)
    return ((x - mean) * mul + np.asarray(bias, F32)).astype(F32)


def gelu(x):
    """flax.linen.gelu (model.py:104), tanh approximation."""
    x = np.asarray(x, F32)
    c = F32(np.sqrt(2.0 / np.pi))
    return (x * (F32(0.5) * (F32(1) + np.tanh(c * (x + F32(0.044715) * (x * x * x)))))).astype(F32)


def _proj(x, p):
    """DenseGeneral d_model -> [heads, head_dim] (query / key / value)."""
    k = np.asarray(p["kernel"], F32)
    return (np.einsum("...m,mhd->...hd", x, k) + np.asarray(p["bias"], F32)).astype(F32)


def _out(a, p):
    """DenseGeneral [heads, head_dim] -> d_model."""
    return (np.einsum("...hd,hdm->...m", a, np.asarray(p["kernel"], F32)) + np.asarray(p["bias"], F32)).astype(F32)


def attention(h, p, n_heads):
    """Causal self-attention over [B, T, d_model] (model.py:88-95)."""
    q, k, v = _proj(h, p["query"]), _proj(h, p["key"]), _proj(h, p["value"])   # [B, T, H, dh]
    dh = q.shape[-1]
    q = (q / np.sqrt(F32(dh))).astype(F32)
    s = np.einsum("bqhd,bkhd->bhqk", q, k).astype(F32)
    T = h.shape[1]
    causal = np.tril(np.ones((T, T), bool))
    s = np.where(causal, s, np.finfo(F32).min)
    w = ml.softmax(s, axis=-1)
    a = np.einsum("bhqk,bkhd->bqhd", w, v).astype(F32)
    return _out(a, p["out"])


def _block_tail(cfg: ModelCfg, params, i, x, h, **pool_kw):
    """The feed-forward / memory half of layer i (model.py:96-121): returns y."""
    P = cfg.pool
    is_mem = i in cfg.memory_layers
    y = np.zeros_like(x)
    if not is_mem or cfg.memory_ffn:
        f = ml.dense(h, params[f"ffn_in_{i}"]["kernel"], params[f"ffn_in_{i}"]["bias"])
        y = ml.dense(gelu(f), params[f"ffn_out_{i}"]["kernel"], params[f"ffn_out_{i}"]["bias"])
    if is_mem:
        lead = h.shape[:-1]
        hh = h.reshape(-1, cfg.d_model)
        pool = params["pool"]
        ym, _, _ = ml.layer_forward(P, hh, params[f"router_{i}"]["kernel"], params[f"router_{i}"]["bias"],
                                    pool["sub_keys"], pool["log_temperature"], pool["values"],
                                    params[f"mem_gate_{i}"]["kernel"], params[f"mem_gate_{i}"]["bias"],
                                    params[f"mem_out_{i}"]["kernel"], params[f"mem_out_{i}"]["bias"], **pool_kw)
        y = (y + ym.reshape(*lead, cfg.d_model)).astype(F32)
    return y


def forward(cfg: ModelCfg, params: Dict, tokens: np.ndarray, **pool_kw) -> np.ndarray:
    """MemoryPoolLM.__call__ (model.py:41-127), train=False: logits [B, T, V]."""
    tokens = np.asarray(tokens)
    B, T = tokens.shape
    E = np.asarray(params["embed"]["embedding"], F32)
    x = (E[tokens] + np.asarray(params["pos_embed"], F32)[None, :T]).astype(F32)   # model.py:61-66
    for i in range(cfg.n_layers):
        h = layer_norm(x, **params[f"ln_attn_{i}"])                                 # model.py:87
        x = (x + attention(h, params[f"attn_{i}"], cfg.n_heads)).astype(F32)        # model.py:88-95
        h = layer_norm(x, **params[f"ln_ffn_{i}"])                                  # model.py:96
        x = (x + _block_tail(cfg, params, i, x, h, **pool_kw)).astype(F32)           # model.py:97-121
    x = layer_norm(x, **params["ln_final"])                                         # model.py:124
    return (x @ E.T).astype(F32)                                                    # model.py:125


def empty_cache(cfg: ModelCfg, batch: int) -> Dict[str, np.ndarray]:
    """Key / value cache of every layer: [L, B, max_len, H, head_dim]."""
    dh = cfg.d_model // cfg.n_heads
    shape = (cfg.n_layers, batch, cfg.max_len, cfg.n_heads, dh)
    return {"key": np.zeros(shape, F32), "value": np.zeros(shape, F32)}


def decode_step(cfg: ModelCfg, params: Dict, cache: Dict, tokens: np.ndarray, pos: int, **pool_kw) -> np.ndarray:
    """One decode step (generate.py:31-34 with MemoryPoolLM(decode=True)):
    tokens [B] at position pos -> logits [B, V]; the cache is updated in place."""
    tokens = np.asarray(tokens)
    E = np.asarray(params["embed"]["embedding"], F32)
    x = (E[tokens] + np.asarray(params["pos_embed"], F32)[pos][None]).astype(F32)   # [B, dm], model.py:63-64
    for i in range(cfg.n_layers):
        p = params[f"attn_{i}"]
        h = layer_norm(x, **params[f"ln_attn_{i}"])
        q, k, v = _proj(h, p["query"]), _proj(h, p["key"]), _proj(h, p["value"])   # [B, H, dh]
        cache["key"][i, :, pos] = k
        cache["value"][i, :, pos] = v
        dh = q.shape[-1]
        q = (q / np.sqrt(F32(dh))).astype(F32)
        K, V = cache["key"][i], cache["value"][i]                                   # [B, max_len, H, dh]
        s = np.einsum("bhd,bkhd->bhk", q, K).astype(F32)
        s = np.where(np.arange(cfg.max_len)[None, None, :] <= pos, s, np.finfo(F32).min)
        w = ml.softmax(s, axis=-1)
        a = np.einsum("bhk,bkhd->bhd", w, V).astype(F32)
        x = (x + _out(a, p["out"])).astype(F32)
        h = layer_norm(x, **params[f"ln_ffn_{i}"])
        x = (x + _block_tail(cfg, params, i, x, h, **pool_kw)).astype(F32)
    x = layer_norm(x, **params["ln_final"])
    return (x @ E.T).astype(F32)


def generate(cfg: ModelCfg, params: Dict, prompt: np.ndarray, n_new: int) -> Dict[str, np.ndarray]:
    """Generator.generate (generate.py:36-63), greedy (temperature 0)."""
    prompt = np.asarray(prompt, np.int32)
    B, P = prompt.shape
    if P + n_new > cfg.max_len:
        raise ValueError("prompt + n_new exceeds max_len")
    cache = empty_cache(cfg, B)
    tok = prompt[:, 0]
    out, logits_all = [], []
    for pos in range(P + n_new - 1):
        logits = decode_step(cfg, params, cache, tok, pos)
        nxt = prompt[:, pos + 1] if pos + 1 < P else np.argmax(logits, -1).astype(np.int32)
        logits_all.append(logits)
        if pos + 1 >= P:
            out.append(nxt)
        tok = nxt
    return {"tokens": np.stack(out, 1) if out else np.zeros((B, 0), np.int32), "logits": np.stack(logits_all, 1)}


def init_params(cfg: ModelCfg, seed: int = 0, values_std: Optional[float] = None) -> Dict:
    """Seeded parameters with the reference's shapes and initialisers' scales
    (nn.Embed: normal(1); pos_embed: normal(0.02); Dense / DenseGeneral:
    lecun normal kernels, zero biases; LayerNorm: ones / zeros; the pool as
    memory.py:99-113)."""
    rng = np.random.default_rng(seed)
    dm, H = cfg.d_model, cfg.n_heads
    dh = dm // H
    P = cfg.pool

    def lecun(fan_in, *shape):
        return (rng.standard_normal(shape) / np.sqrt(fan_in)).astype(F32)

    def dense(fi, fo):
        return {"kernel": lecun(fi, fi, fo), "bias": (rng.standard_normal(fo) * 0.02).astype(F32)}

    def ln():
        return {"scale": (1 + 0.1 * rng.standard_normal(dm)).astype(F32),
                "bias": (0.05 * rng.standard_normal(dm)).astype(F32)}

    p = {"embed": {"embedding": rng.standard_normal((cfg.vocab_size, dm)).astype(F32)},
         "pos_embed": (rng.standard_normal((cfg.max_len, dm)) * 0.02).astype(F32)}
    for i in range(cfg.n_layers):
        p[f"ln_attn_{i}"] = ln()
        p[f"attn_{i}"] = {n: {"kernel": lecun(dm, dm, H, dh), "bias": (rng.standard_normal((H, dh)) * 0.02).astype(F32)}
                          for n in ("query", "key", "value")}
        p[f"attn_{i}"]["out"] = {"kernel": lecun(dm, H, dh, dm), "bias": (rng.standard_normal(dm) * 0.02).astype(F32)}
        p[f"ln_ffn_{i}"] = ln()
        if i not in cfg.memory_layers or cfg.memory_ffn:
            p[f"ffn_in_{i}"] = dense(dm, dm * cfg.ffn_mult)
            p[f"ffn_out_{i}"] = dense(dm * cfg.ffn_mult, dm)
        if i in cfg.memory_layers:
            p[f"router_{i}"] = dense(dm, P.heads * P.d_key)
            p[f"mem_gate_{i}"] = dense(dm, P.d_value)
            p[f"mem_out_{i}"] = dense(P.d_value, dm)
    sk = rng.standard_normal((P.heads, 2, P.n_sub_keys, P.d_key // 2)).astype(F32)
    std = P.d_value ** -0.5 if values_std is None else values_std
    p["pool"] = {"sub_keys": ml.l2_normalize(sk), "values": (rng.standard_normal((P.pool_size, P.d_value)) * std)
                 .astype(F32), "log_temperature": F32(np.log(P.init_temperature))}
    p["ln_final"] = ln()
    return p
