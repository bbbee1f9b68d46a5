"""Deterministic synthetic inputs for the golden fixtures and parity tests.

Large inputs are not stored in the fixtures: they are regenerated from a
counter-based hash (splitmix64 over ``seed`` and the flat element index), so
a fixture only needs its recipe and the expected outputs.  The same recipe
runs here and on the GPU box and gives the same float32 arrays.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def _splitmix64(x: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = x + np.uint64(0x9E3779B97F4A7C15)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def _hash_u01(n: int, seed: int) -> np.ndarray:
    """float64 uniform in [0, 1) (53-bit) from splitmix64(seed, index)."""
    with np.errstate(over="ignore"):
        base = np.uint64(seed) * np.uint64(0xD1B54A32D192ED03)
        x = _splitmix64(np.arange(n, dtype=np.uint64) + base)
    return (x >> np.uint64(11)).astype(np.float64) * (1.0 / 9007199254740992.0)


def hash_uniform(shape, seed: int, lo: float = 0.0, hi: float = 1.0) -> np.ndarray:
    """float32 uniform in [lo, hi) from splitmix64(seed, index)."""
    u = _hash_u01(int(np.prod(shape)), seed)
    return np.minimum(lo + (hi - lo) * u, np.nextafter(F32(hi), F32(lo))).astype(F32).reshape(shape)


def hash_normal(shape, seed: int, std: float = 1.0, mean: float = 0.0) -> np.ndarray:
    """float32 normal via Box-Muller over two float64 hash-uniform streams."""
    n = int(np.prod(shape))
    u1 = _hash_u01(n, seed * 2 + 1)
    u2 = _hash_u01(n, seed * 2 + 2)
    z = np.sqrt(-2.0 * np.log1p(-u1)) * np.cos(2.0 * np.pi * u2)
    return (mean + std * z).astype(F32).reshape(shape)


def glorot_uniform(fan_in: int, fan_out: int, seed: int) -> np.ndarray:
    """flax default Dense kernel init (lecun normal) is replaced by the
    Glorot-uniform init the benchmark configs name."""
    lim = np.sqrt(6.0 / (fan_in + fan_out))
    return hash_uniform((fan_in, fan_out), seed, -lim, lim)


def round_fp16(x: np.ndarray) -> np.ndarray:
    """float32 -> float16 -> float32 (round to nearest even)."""
    return np.asarray(x, F32).astype(np.float16).astype(F32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """float32 -> bfloat16 -> float32 (round to nearest even, NaN kept)."""
    b = np.asarray(x, F32).view(np.uint32).astype(np.uint64)
    rounded = (b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) & np.uint64(0xFFFF0000)
    return rounded.astype(np.uint32).view(F32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """uint16 bit patterns of round_bf16(x)."""
    return (round_bf16(x).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def clustered_hidden(T: int, d: int, seed: int, n_centers: int = 64, sigma: float = 0.3,
                     zipf_a: float = 1.1) -> np.ndarray:
    """Hidden states drawn from ``n_centers`` Gaussian clusters whose
    weights follow Zipf(zipf_a) (p_r proportional to r^-a, r = 1..n_centers),
    as in the billion-slot and sparse-update benchmark configs."""
    centers = hash_normal((n_centers, d), seed * 7 + 3)
    p = np.arange(1, n_centers + 1, dtype=np.float64) ** -zipf_a
    cdf = np.cumsum(p / p.sum())
    u = hash_uniform((T,), seed * 7 + 4).astype(np.float64)
    c = np.minimum(np.searchsorted(cdf, u, side="right"), n_centers - 1)
    return (centers[c] + sigma * hash_normal((T, d), seed * 7 + 5)).astype(F32)


def pool_inputs(recipe: dict) -> dict:
    """Regenerate every input array of a golden case from its recipe."""
    n, H, dk, dv, M = (recipe[k] for k in ("n_sub_keys", "heads", "d_key", "d_value", "M"))
    half = dk // 2
    s = recipe["seed"]
    out = {}
    if recipe.get("layer", False):
        dm = recipe["d_model"]
        out["h"] = (clustered_hidden(M, dm, s + 11) if recipe.get("clustered")
                    else hash_normal((M, dm), s + 11))
        out["w_router"] = glorot_uniform(dm, H * dk, s + 12)
        out["b_router"] = hash_normal((H * dk,), s + 13, 0.01) if recipe.get("biases") else np.zeros(H * dk, F32)
        out["w_gate"] = glorot_uniform(dm, dv, s + 14)
        out["b_gate"] = hash_normal((dv,), s + 15, 0.01) if recipe.get("biases") else np.zeros(dv, F32)
        out["w_out"] = glorot_uniform(dv, dm, s + 16)
        out["b_out"] = hash_normal((dm,), s + 17, 0.01) if recipe.get("biases") else np.zeros(dm, F32)
    else:
        out["queries"] = hash_normal((M, H, dk), s + 1)
    out["sub_keys"] = hash_normal((H, 2, n, half), s + 2, recipe.get("key_std", 1.0))
    if recipe.get("tie_keys"):
        # duplicated sub-keys: exact ties in every cosine score against them
        sk = out["sub_keys"]
        sk[:, :, 1::2] = sk[:, :, 0::2]
        out["sub_keys"] = sk
    v = hash_normal((n * n, dv), s + 3, recipe.get("value_std", 0.02))
    if recipe.get("values_dtype") == "fp16":
        v = round_fp16(v)
    elif recipe.get("values_dtype") == "bf16":
        v = round_bf16(v)
    out["values"] = v
    out["log_t"] = F32(recipe.get("log_t", float(np.log(F32(10.0)))))
    if recipe.get("noise", 0.0) > 0:
        u = np.maximum(_hash_u01(M * H * 2 * n, s + 4), 1e-12).reshape(M, H, 2, n)
        out["gumbel"] = (-np.log(-np.log(u))).astype(F32)
    return out
