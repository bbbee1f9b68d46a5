"""CPU oracle for the memory-layer hot path (TEST INFRASTRUCTURE ONLY).

This module is a float32 numpy restatement of the reference memory layer of
KumarDev7/model:

* ``memory_pool_model/memory.py:30-57``   l2-normalise and top-k helpers
* ``memory_pool_model/memory.py:119-227`` ``MemoryPool.__call__``
* ``memory_pool_model/model.py:108-120``  router Dense, SiLU gate, output Dense, and
  the gradients through that block (``layer_backward``)
* ``memory_pool_model/train.py:146-206``  fetched-row gradients (unique + segment sum),
  single device and data-parallel (local merge, all-gather, second merge)
* ``memory_pool_model/train.py:396-416``  global-norm clip + row-wise Adagrad
* ``memory_pool_model/memory.py:230-281`` ``key_diversity_loss`` (with its
  gradient) and ``revive_dead_keys`` (random draws passed in)

It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import
it.  The product path (``model_b200``) never calls into this file.

Pinning.  The reference's arithmetic lives in JAX/XLA, which is not installed
in this environment.  The oracle is pinned against golden vectors produced by
running the reference's own ``memory.py`` source over a numpy restatement of
the JAX primitives it calls (``tests/golden/make_golden.py``), and against
restatements of the reference's property tests
(``tests/test_memory_pool.py``).  JAX's own float32 accumulation order is not
pinned; every comparison therefore allows float32 re-association error.
"""

from __future__ import annotations

import dataclasses
from typing import Dict, Optional, Tuple

import numpy as np

F32 = np.float32


# --------------------------------------------------------------------------
# helpers (memory.py:30-57)
# --------------------------------------------------------------------------
def l2_normalize(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """memory.py:30-31: x * rsqrt(sum(x*x) + eps) over the last axis."""
    x = np.asarray(x, F32)
    ss = np.sum(x * x, axis=-1, keepdims=True, dtype=F32) + F32(eps)
    return (x * (F32(1.0) / np.sqrt(ss))).astype(F32)


def top_k(x: np.ndarray, k: int) -> Tuple[np.ndarray, np.ndarray]:
    """Top-k over the last axis with lax.top_k semantics (memory.py:34-57).

    Values are sorted descending; equal values are ordered lowest index
    first, which is what both ``_top_k_by_max`` (repeated first-argmax,
    memory.py:34-45) and ``lax.top_k`` (memory.py:56) return.
    """
    x = np.asarray(x)
    n = x.shape[-1]
    if not 0 < k <= n:
        raise ValueError(f"top_k: k={k} must be in [1, {n}]")
    flat = x.reshape(-1, n)
    if k == n:
        sel = np.broadcast_to(np.arange(n), flat.shape)
    else:
        # any k elements holding the k largest values ...
        sel = np.argpartition(-flat, k - 1, axis=-1)[:, :k]
        thr = np.take_along_axis(flat, sel, axis=-1).min(-1, keepdims=True)
        # ... which is the lax.top_k set unless the k-th value is tied with
        # an element left out; those rows take the lowest-index tied elements
        amb = np.flatnonzero((flat == thr).sum(-1) > (np.take_along_axis(flat, sel, -1) == thr).sum(-1))
        if amb.size:
            f, t = flat[amb], thr[amb]
            gt, eq = f > t, f == t
            take = gt | (eq & (np.cumsum(eq, axis=-1) <= k - gt.sum(-1, keepdims=True)))
            sel = sel.copy()
            sel[amb] = np.nonzero(take)[1].reshape(amb.size, k)
        sel = np.sort(sel, axis=-1)
    vals = np.take_along_axis(flat, sel, axis=-1)
    # stable sort on the negated values keeps ascending index among ties
    order = np.argsort(-vals, axis=-1, kind="stable")
    idx = np.take_along_axis(sel, order, axis=-1)
    vals = np.take_along_axis(vals, order, axis=-1)
    return vals.reshape(*x.shape[:-1], k), idx.reshape(*x.shape[:-1], k).astype(np.int32)


def temperature(log_t: float, min_t: float, max_t: float) -> np.float32:
    """memory.py:141-146: straight-through clamp of log T, forward value."""
    log_t = F32(log_t)
    lo, hi = np.log(F32(min_t)), np.log(F32(max_t))
    clipped = np.clip(log_t, lo, hi).astype(F32)
    return np.exp(F32(log_t + F32(clipped - log_t))).astype(F32)


def softmax(x: np.ndarray, axis: int = -1) -> np.ndarray:
    """jax.nn.softmax: exp(x - max) / sum(exp(x - max))."""
    x = np.asarray(x, F32)
    e = np.exp(x - np.max(x, axis=axis, keepdims=True))
    return (e / np.sum(e, axis=axis, keepdims=True, dtype=F32)).astype(F32)


def silu(x: np.ndarray) -> np.ndarray:
    """flax.linen.silu (model.py:118): x * sigmoid(x)."""
    x = np.asarray(x, F32)
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


# --------------------------------------------------------------------------
# MemoryPool (memory.py:64-227)
# --------------------------------------------------------------------------
@dataclasses.dataclass(frozen=True)
class PoolConfig:
    """The MemoryPool fields of memory.py:72-97 (config.py:35-59)."""

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

    @property
    def pool_size(self) -> int:
        return self.n_sub_keys ** 2


def route(cfg: PoolConfig, queries: np.ndarray, sub_keys: np.ndarray, log_t: float,
          train: bool = False, gumbel: Optional[np.ndarray] = None, noise_scale: float = 1.0):
    """Routing half of memory.py:132-175.

    Returns a dict with q (unit query halves [M,H,2,half]), q_len, cos,
    scores, select_scores, sub_idx [M,H,2,k], slot_scores [M,H,k],
    slots [M,H,k], idx_a, idx_b and the temperature.
    ``gumbel`` is the standard Gumbel sample the reference draws from the
    "routing" RNG stream (memory.py:156); it is an explicit input here.
    """
    H, n, k = cfg.heads, cfg.n_sub_keys, cfg.top_k
    half = cfg.d_key // 2
    q = np.asarray(queries, F32).reshape(-1, H, 2, half)               # memory.py:136
    q_len = (np.sqrt(np.sum(q * q, axis=-1, keepdims=True, dtype=F32) + F32(1e-6))
             / np.sqrt(F32(half))).astype(F32)                          # memory.py:137
    qn = l2_normalize(q)                                                # memory.py:138
    keys = l2_normalize(sub_keys)                                       # memory.py:139
    T = temperature(log_t, cfg.min_temperature, cfg.max_temperature)    # memory.py:143-146
    M = q.shape[0]
    cos = np.empty((M, H, 2, n), F32)
    for h in range(H):                                                  # memory.py:149
        for c in range(2):
            cos[:, h, c, :] = qn[:, h, c, :] @ keys[h, c].T
    scores = (cos * T).astype(F32)                                      # memory.py:150
    if cfg.query_scale:
        scores = (scores * q_len).astype(F32)                           # memory.py:151-152
    if train and cfg.routing_noise > 0 and gumbel is not None:          # memory.py:155-159
        coef = F32(cfg.routing_noise * noise_scale)
        select = (scores + coef * np.asarray(gumbel, F32)).astype(F32)
    else:
        select = scores
    _, sub_idx = top_k(select, k)                                       # memory.py:162
    sub_scores = np.take_along_axis(scores, sub_idx, axis=-1)           # memory.py:163
    sub_select = np.take_along_axis(select, sub_idx, axis=-1)           # memory.py:164
    cand = (sub_scores[..., 0, :, None] + sub_scores[..., 1, None, :]).reshape(M, H, k * k)
    cand_sel = (sub_select[..., 0, :, None] + sub_select[..., 1, None, :]).reshape(M, H, k * k)
    _, flat_idx = top_k(cand_sel, k)                                    # memory.py:171
    slot_scores = np.take_along_axis(cand, flat_idx, axis=-1)           # memory.py:172
    idx_a = np.take_along_axis(sub_idx[..., 0, :], flat_idx // k, axis=-1)
    idx_b = np.take_along_axis(sub_idx[..., 1, :], flat_idx % k, axis=-1)
    slots = (idx_a.astype(np.int64) * n + idx_b).astype(np.int64)       # memory.py:175
    return dict(q=qn, q_len=q_len, cos=cos, scores=scores, select=select, sub_idx=sub_idx,
                sub_scores=sub_scores, slot_scores=slot_scores, slots=slots,
                idx_a=idx_a, idx_b=idx_b, temperature=T)


def gather_mix(values: np.ndarray, slots: np.ndarray, weights: np.ndarray,
               shuffle_reads: bool = False, chunk: int = 2048) -> np.ndarray:
    """memory.py:179-192: out[m] = sum_h sum_k w[m,h,k] * values[read_slot].

    ``values`` may be float16/bfloat16-rounded storage; rows are upcast to
    float32 on read as in host_pool.py:120.  Work is chunked over tokens so
    the [M,H,k,d] fetched tensor is never materialised whole.
    """
    N = values.shape[0]
    read = (slots + N // 2 + 1) % N if shuffle_reads else slots         # memory.py:179
    M = slots.shape[0]
    out = np.empty((M, values.shape[1]), F32)
    for s in range(0, M, chunk):
        rows = np.asarray(values[read[s:s + chunk]], F32)                # [m,H,k,d]
        out[s:s + chunk] = np.einsum("mhk,mhkd->md", weights[s:s + chunk], rows,
                                     optimize=True).astype(F32)          # memory.py:192
    return out


def pool_forward(cfg: PoolConfig, queries: np.ndarray, sub_keys: np.ndarray, log_t: float,
                 values: np.ndarray, *, train: bool = False, gumbel: Optional[np.ndarray] = None,
                 noise_scale: float = 1.0, shuffle_reads: bool = False,
                 with_stats: bool = True) -> Tuple[np.ndarray, Dict[str, np.ndarray]]:
    """MemoryPool.__call__ (memory.py:119-227): returns (out [..., d], aux)."""
    lead = np.asarray(queries).shape[:-2]
    H, n, k = cfg.heads, cfg.n_sub_keys, cfg.top_k
    r = route(cfg, queries, sub_keys, log_t, train, gumbel, noise_scale)
    weights = softmax(r["slot_scores"])                                 # memory.py:178
    out = gather_mix(values, r["slots"], weights, shuffle_reads)
    aux = dict(slots=r["slots"].reshape(*lead, H, k), weights=weights.reshape(*lead, H, k),
               temperature=r["temperature"], queries=r["q"],
               top1_weight=F32(weights.max(-1).mean(dtype=np.float64)))
    if with_stats:
        aux.update(pool_stats(cfg, r, train and cfg.routing_noise > 0 and gumbel is not None))
    return out.reshape(*lead, cfg.d_value), aux


def pool_stats(cfg: PoolConfig, r: Dict[str, np.ndarray], noisy: bool) -> Dict[str, np.ndarray]:
    """Routing statistics of memory.py:196-215."""
    H, n, k = cfg.heads, cfg.n_sub_keys, cfg.top_k
    M = r["q"].shape[0]
    codebook = (np.arange(H)[:, None, None] * 2 + np.arange(2)[None, :, None]) * n

    def count_subkeys(ids):                                             # memory.py:200-202
        flat = (ids + codebook).reshape(-1)
        return np.bincount(flat, minlength=H * 2 * n).astype(F32).reshape(H, 2, n)

    subkey_counts = count_subkeys(np.stack([r["idx_a"], r["idx_b"]], axis=2))
    clean_idx = top_k(r["scores"], k)[1] if noisy else r["sub_idx"]     # memory.py:208
    f = (count_subkeys(clean_idx) / F32(M * k)).astype(F32)
    if cfg.balance_temperature_grad:                                    # memory.py:211
        p_scores = r["scores"]
    else:
        p_scores = (r["cos"] * r["temperature"]).astype(F32)
    P = softmax(p_scores).mean(axis=0, dtype=np.float64).astype(F32)    # memory.py:212
    balance_loss = F32(n * np.mean(np.sum(f.astype(np.float64) * P, axis=-1)))
    slot_counts = np.bincount(r["slots"].reshape(-1), minlength=cfg.pool_size).astype(F32)
    return dict(subkey_counts=subkey_counts, slot_counts=slot_counts,
                balance_loss=balance_loss, balance_P=P, balance_f=f)


# --------------------------------------------------------------------------
# Memory layer block (model.py:108-120)
# --------------------------------------------------------------------------
def dense(x: np.ndarray, kernel: np.ndarray, bias: Optional[np.ndarray]) -> np.ndarray:
    """flax.linen.Dense: x @ kernel + bias (float32)."""
    y = np.asarray(x, F32) @ np.asarray(kernel, F32)
    if bias is not None:
        y = y + np.asarray(bias, F32)
    return y.astype(F32)


def layer_forward(cfg: PoolConfig, h: np.ndarray, w_router, b_router, sub_keys, log_t, values,
                  w_gate, b_gate, w_out, b_out, *, train=False, gumbel=None, noise_scale=1.0,
                  shuffle_reads=False, with_stats=False):
    """model.py:110-119 for one memory layer, given the normalised hidden h [T, d_model].

    Returns (y_mem [T, d_model], mem [T, d_value], aux) where y_mem is the
    term the reference adds into ``y`` (model.py:119).
    """
    T = h.shape[0]
    q = dense(h, w_router, b_router).reshape(T, cfg.heads, cfg.d_key)    # model.py:110-111
    mem, aux = pool_forward(cfg, q, sub_keys, log_t, values, train=train, gumbel=gumbel,
                            noise_scale=noise_scale, shuffle_reads=shuffle_reads,
                            with_stats=with_stats)                     # model.py:112-113
    gate = silu(dense(h, w_gate, b_gate))                               # model.py:118
    y = dense((mem * gate).astype(F32), w_out, b_out)                   # model.py:119
    return y, mem, aux


def layer_backward(cfg: PoolConfig, h, w_router, b_router, sub_keys, log_t, values, w_gate, b_gate, w_out,
                   b_out, dy, *, balance_coef: float = 0.0, route_through_pool: bool = False,
                   train: bool = False, gumbel=None, noise_scale: float = 1.0, shuffle_reads: bool = False):
    """Gradients of sum(dy * y) + balance_coef * balance_loss through one
    memory layer (model.py:110-119 with memory.py:133-214), as the reference
    trainer's jax.value_and_grad computes them with sparse_grad (the value
    table gets none; its rows' gradient is the read-output gradient
    ``probe``, model.py:114-115).  Routing (top-k indices) comes from the
    float32 forward and carries no gradient; the temperature clamp is
    straight-through (memory.py:141-146); the balance term reaches every
    sub-key through the softmax over all keys (memory.py:210-214).
    route_through_pool: the gate reads stop_gradient(h) (model.py:116-117).
    Computed in float64.  Returns a dict of float64 arrays: h, w_router,
    b_router, sub_keys, log_temperature, w_gate, b_gate, w_out, b_out, probe
    ([T, d_value]), plus the forward's slots and weights."""
    f64 = np.float64
    H, n, k = cfg.heads, cfg.n_sub_keys, cfg.top_k
    half = cfg.d_key // 2
    T_ = h.shape[0]
    q_raw = dense(h, w_router, b_router).reshape(T_, H, cfg.d_key)
    r = route(cfg, q_raw, sub_keys, log_t, train, gumbel, noise_scale)
    w = softmax(r["slot_scores"]).astype(f64)                                # memory.py:178
    N = cfg.pool_size
    read = (r["slots"] + N // 2 + 1) % N if shuffle_reads else r["slots"]    # memory.py:179
    V = np.asarray(values, f64)
    fetched = V[read]                                                        # [T, H, k, d]
    mem = np.einsum("mhk,mhkd->md", w, fetched)                              # memory.py:192
    hh = np.asarray(h, f64)
    zg = hh @ np.asarray(w_gate, f64) + (0.0 if b_gate is None else np.asarray(b_gate, f64))
    sig = 1.0 / (1.0 + np.exp(-zg))
    gate = zg * sig                                                          # model.py:118
    dy = np.asarray(dy, f64)
    out = {}
    # model.py:119  y = (mem * gate) W_out + b_out
    memg = mem * gate
    out["w_out"] = memg.T @ dy
    out["b_out"] = dy.sum(0)
    dmemg = dy @ np.asarray(w_out, f64).T
    dmem = dmemg * gate
    out["probe"] = dmem                                                      # model.py:114-115
    dgate = dmemg * mem
    dzg = dgate * sig * (1.0 + zg * (1.0 - sig))                             # silu'
    out["w_gate"] = hh.T @ dzg
    out["b_gate"] = dzg.sum(0)
    dh = np.zeros_like(hh) if route_through_pool else dzg @ np.asarray(w_gate, f64).T
    # memory.py:192  d weights = dmem . fetched row, then the softmax (:178)
    dw = np.einsum("md,mhkd->mhk", dmem, fetched)
    dss = w * (dw - np.sum(w * dw, axis=-1, keepdims=True))
    # memory.py:166-172  slot score = scores[0, idx_a] + scores[1, idx_b]
    dscores = np.zeros((T_, H, 2, n), f64)
    mi = np.arange(T_)[:, None, None]
    hi = np.arange(H)[None, :, None]
    np.add.at(dscores, (mi, hi, 0, r["idx_a"]), dss)
    np.add.at(dscores, (mi, hi, 1, r["idx_b"]), dss)
    Tv = f64(r["temperature"])
    cos = np.asarray(r["cos"], f64)
    qn = np.asarray(r["q"], f64)
    q_len = np.asarray(r["q_len"], f64)
    # memory.py:205-214  balance_loss = n * mean_{h,c} sum_i f_i P_i
    dcos_bal = np.zeros_like(cos)
    if balance_coef != 0.0:
        st = pool_stats(cfg, r, train and cfg.routing_noise > 0 and gumbel is not None)
        fcount = np.asarray(st["balance_f"], f64)                             # [H, 2, n], no gradient
        dP = balance_coef * n / (H * 2) * fcount
        p = np.asarray(r["scores"], f64) if cfg.balance_temperature_grad else cos * Tv
        p = p - p.max(-1, keepdims=True)
        sm = np.exp(p)
        sm /= sm.sum(-1, keepdims=True)
        dp = sm * (dP[None] - np.sum(sm * dP[None], axis=-1, keepdims=True)) / T_
        if cfg.balance_temperature_grad:
            dscores += dp
        else:
            dcos_bal = dp * Tv                                               # sg(T): no temperature gradient
    # memory.py:150-152  scores = cos * T (* q_len)
    scale = Tv * (q_len if cfg.query_scale else 1.0)
    dcos = dscores * scale + dcos_bal
    dT = np.sum(dscores * cos * (q_len if cfg.query_scale else 1.0))
    out["log_temperature"] = dT * Tv                                         # straight-through clamp
    dq_len = np.sum(dscores * cos * Tv, axis=-1, keepdims=True) if cfg.query_scale else 0.0
    # memory.py:149  cos = q_hat . k_hat
    keys_n = np.asarray(l2_normalize(sub_keys), f64)
    dqn = np.einsum("mhcn,hcnd->mhcd", dcos, keys_n)
    dkn = np.einsum("mhcn,mhcd->hcnd", dcos, qn)
    # memory.py:136-138, 139  normalisation backward (x * rsqrt(|x|^2 + 1e-6))
    q = q_raw.reshape(T_, H, 2, half).astype(f64)
    rq = 1.0 / np.sqrt(np.sum(q * q, -1, keepdims=True) + 1e-6)
    dq = rq * dqn - rq ** 3 * np.sum(q * dqn, -1, keepdims=True) * q
    if cfg.query_scale:
        dq = dq + dq_len * q * rq / np.sqrt(half)
    x = np.asarray(sub_keys, f64)
    rk = 1.0 / np.sqrt(np.sum(x * x, -1, keepdims=True) + 1e-6)
    out["sub_keys"] = rk * dkn - rk ** 3 * np.sum(x * dkn, -1, keepdims=True) * x
    dq = dq.reshape(T_, H * cfg.d_key)
    out["w_router"] = hh.T @ dq                                              # model.py:110
    out["b_router"] = dq.sum(0)
    out["h"] = dh + dq @ np.asarray(w_router, f64).T
    out["slots"] = r["slots"]
    out["weights"] = w.astype(F32)
    return out


# --------------------------------------------------------------------------
# Sparse row gradients + row-wise Adagrad (train.py:146-172, 396-416)
# --------------------------------------------------------------------------
def fetched_row_grads(slots: np.ndarray, weights: np.ndarray, g_out: np.ndarray, pool_size: int):
    """train.py:146-172: (uniq [U], rows [U, d]) with rows[u] = sum over
    fetches f of slot uniq[u] of w_f * dL/dout[token(f)].  Only the U
    distinct fetched slots are returned (no padding)."""
    M = g_out.shape[0]
    sl = slots.reshape(M, -1).reshape(-1)
    w = weights.reshape(M, -1).astype(F32)
    contrib = (w[..., None] * g_out[:, None, :]).reshape(-1, g_out.shape[-1]).astype(F32)
    uniq, inv = np.unique(sl, return_inverse=True)
    rows = np.zeros((uniq.shape[0], g_out.shape[-1]), F32)
    np.add.at(rows, inv.reshape(-1), contrib)
    return uniq.astype(np.int64), rows


def fetched_row_grads_sharded(per_device, pool_size: int):
    """train.py:175-206: every device merges its own fetches
    (fetched_row_grads), the devices' merged (uniq, rows) are concatenated in
    device order (the tiled all_gather) and merged once more (_merge_rows,
    train.py:160-172: unique + segment sum in concatenation order).
    per_device = [(slots, weights, g_out), ...]; a device with no tokens
    passes empty arrays."""
    us, rs = [], []
    d = None
    for slots, weights, g_out in per_device:
        d = g_out.shape[-1]
        if g_out.shape[0] == 0:
            continue
        u, r = fetched_row_grads(slots, weights, g_out, pool_size)
        us.append(u)
        rs.append(r)
    if not us:
        return np.zeros(0, np.int64), np.zeros((0, d), F32)
    u_all = np.concatenate(us)
    r_all = np.concatenate(rs).astype(F32)
    uniq, inv = np.unique(u_all, return_inverse=True)
    rows = np.zeros((uniq.shape[0], r_all.shape[1]), F32)
    np.add.at(rows, inv.reshape(-1), r_all)
    return uniq.astype(np.int64), rows


def rowwise_adagrad(values: np.ndarray, acc: np.ndarray, uniq: np.ndarray, g_rows: np.ndarray,
                    lr: float) -> None:
    """train.py:412-416 in place: acc[u] += mean(g^2); V[u] -= lr/(sqrt(acc)+1e-8) * g."""
    a = (acc[uniq] + np.mean(g_rows * g_rows, axis=-1, dtype=F32)).astype(F32)
    step = (F32(lr) / (np.sqrt(a) + F32(1e-8))).astype(F32)
    values[uniq] = (values[uniq] + (-step)[:, None] * g_rows).astype(values.dtype)
    acc[uniq] = a


def clip_scale(g_rest_sq_norm: float, g_rows: np.ndarray, grad_clip: float) -> np.float32:
    """train.py:396-398: min(1, clip / (global_norm + 1e-6))."""
    gnorm = np.sqrt(np.float64(g_rest_sq_norm) + np.sum(g_rows.astype(np.float64) ** 2))
    return F32(min(1.0, grad_clip / (gnorm + 1e-6)))


# --------------------------------------------------------------------------
# Sub-key maintenance (memory.py:230-281)
# --------------------------------------------------------------------------
def key_diversity_loss(sub_keys: np.ndarray):
    """memory.py:230-240: mean squared off-diagonal cosine inside each
    codebook, and its gradient with respect to sub_keys (the loss enters the
    trainer's loss with key_diversity_coef, train.py:327-329).
    Returns (loss float32, grad [H, 2, n, half] float32)."""
    x = np.asarray(sub_keys, F32)
    H, C, n, d = x.shape
    ss = np.sum(x * x, axis=-1, keepdims=True, dtype=F32)
    r = (F32(1.0) / np.sqrt(ss + F32(1e-6))).astype(F32)
    k = (x * r).astype(F32)                                               # memory.py:31
    gram = np.einsum("hcnd,hcmd->hcnm", k, k).astype(F32)
    off = gram * (F32(1.0) - np.eye(n, dtype=F32))
    denom = F32(H * C * n * (n - 1))
    loss = F32(np.sum(off.astype(np.float64) ** 2) / denom)
    # d loss / d k = 4 / denom * off @ k ; then the normalisation's backward
    dk = (F32(4.0) / denom * np.einsum("hcnm,hcmd->hcnd", off, k)).astype(F32)
    dot = np.sum(x * dk, axis=-1, keepdims=True, dtype=F32)
    dx = (r * dk - (r ** 3) * dot * x).astype(F32)
    return loss, dx


def revive_dead_keys(sub_keys: np.ndarray, usage: np.ndarray, queries: np.ndarray, pick: np.ndarray,
                     noise: np.ndarray, threshold: float, noise_scale: float = 0.05):
    """memory.py:243-281 with the random draws passed in: pick [H, 2, n]
    token indices into queries [M, H, 2, half], noise [H, 2, n, half]
    standard normal.  Returns (new_sub_keys, new_usage, dead)."""
    H, C, n, d = sub_keys.shape
    dead = usage < F32(threshold) / F32(n)
    h_idx = np.arange(H)[:, None, None]
    c_idx = np.arange(C)[None, :, None]
    M = np.asarray(queries).shape[0]
    pick = np.asarray(pick, np.int64)
    pick = np.clip(np.where(pick < 0, pick + M, pick), 0, M - 1)         # XLA gather: clamped indices
    rep = np.asarray(queries, F32)[pick, h_idx, c_idx]                    # [H, C, n, d]
    rep = (rep + F32(noise_scale) * np.asarray(noise, F32)).astype(F32)
    rep = l2_normalize(rep)
    new_keys = np.where(dead[..., None], rep, sub_keys).astype(F32)
    new_usage = np.where(dead, F32(1.0) / F32(n), usage).astype(F32)
    new_usage = (new_usage / np.sum(new_usage, axis=-1, keepdims=True, dtype=F32)).astype(F32)
    return new_keys, new_usage, dead

