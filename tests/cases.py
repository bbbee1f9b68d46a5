"""Run the oracle on a golden recipe (inputs regenerated from the recipe)."""

from __future__ import annotations

import functools

import numpy as np

import inputs as gi
from oracle import memlayer_ref as ref


def pool_config(recipe: dict) -> ref.PoolConfig:
    kw = {k: recipe[k] for k in ("n_sub_keys", "heads", "d_key", "d_value", "top_k")}
    kw["routing_noise"] = recipe.get("noise", 0.0)
    for k in ("min_temperature", "max_temperature", "balance_temperature_grad", "query_scale"):
        if k in recipe:
            kw[k] = recipe[k]
    return ref.PoolConfig(**kw)


@functools.lru_cache(maxsize=4)
def _inputs(key):
    import json
    return gi.pool_inputs(json.loads(key))


def case_inputs(recipe: dict) -> dict:
    import json
    return _inputs(json.dumps(recipe, sort_keys=True))


def run_oracle(recipe: dict, with_stats: bool = True):
    """Oracle outputs for a recipe: dict with out, (y), slots, weights, aux, route."""
    cfg = pool_config(recipe)
    x = case_inputs(recipe)
    if recipe.get("layer"):
        M = recipe["M"]
        q = ref.dense(x["h"], x["w_router"], x["b_router"]).reshape(M, cfg.heads, cfg.d_key)
    else:
        q = x["queries"]
    kw = dict(train=recipe.get("train", False), gumbel=x.get("gumbel"),
              noise_scale=recipe.get("noise_scale", 1.0))
    out, aux = ref.pool_forward(cfg, q, x["sub_keys"], x["log_t"], x["values"],
                                shuffle_reads=recipe.get("shuffle_reads", False), with_stats=with_stats, **kw)
    r = ref.route(cfg, q, x["sub_keys"], x["log_t"], **kw)
    res = dict(out=out, slots=aux["slots"], weights=aux["weights"], aux=aux, route=r, q=q)
    if recipe.get("layer"):
        gate = ref.silu(ref.dense(x["h"], x["w_gate"], x["b_gate"]))
        res["y"] = ref.dense((out * gate).astype(np.float32), x["w_out"], x["b_out"])
    return res


def oracle_from_slots(recipe: dict, slots: np.ndarray, weights: np.ndarray) -> dict:
    """The oracle's read output, layer output and routing counts recomputed
    from a given selection (the GPU's own slots and weights): the check of
    everything downstream of routing where a near-tie let the GPU pick
    another slot than the oracle (memory.py:179-192,200-216, model.py:118-119)."""
    cfg = pool_config(recipe)
    x = case_inputs(recipe)
    H, n, k = cfg.heads, cfg.n_sub_keys, cfg.top_k
    s = np.asarray(slots).reshape(-1, H, k).astype(np.int64)
    w = np.asarray(weights).reshape(-1, H, k).astype(np.float32)
    out = ref.gather_mix(x["values"], s, w, recipe.get("shuffle_reads", False))
    base_a = (np.arange(H) * 2 * n)[None, :, None]          # codebook (h, half 0) starts at 2h * n
    ids = np.concatenate([(s // n + base_a).reshape(-1), (s % n + base_a + n).reshape(-1)])
    res = dict(out=out,
               subkey_counts=np.bincount(ids, minlength=H * 2 * n).astype(np.float32).reshape(H, 2, n),
               slot_counts=np.bincount(s.reshape(-1), minlength=n * n).astype(np.float32))
    if recipe.get("layer"):
        gate = ref.silu(ref.dense(x["h"], x["w_gate"], x["b_gate"]))
        res["y"] = ref.dense((out * gate).astype(np.float32), x["w_out"], x["b_out"])
    return res
