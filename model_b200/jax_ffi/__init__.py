"""JAX binding of the memory layer: XLA FFI custom calls over the C ABI.

The reference is JAX / Flax (memory_pool_model/memory.py:64-227,
model.py:108-120).  ``memlayer_xla.cc`` defines three XLA FFI handlers over
``include/memlayer.h``; this module builds them against
``jax.ffi.include_dir()``, registers them as CUDA custom-call targets and
offers the calls the reference makes:

* :func:`pool_forward` -- ``MemoryPool.__call__`` (memory.py:119-227);
* :func:`memory_block` -- the memory-layer block of model.py:110-119 as a
  ``jax.custom_vjp`` (forward: ``memlayer_layer_forward``; backward:
  ``memlayer_layer_backward``, which returns the read-output gradient
  ``probe`` the sparse row update consumes, train.py:146-172).

JAX is imported lazily: without it, :func:`build` reports that it skipped
the handler library and the other functions raise ImportError.
"""

from __future__ import annotations

import ctypes as C
import math
import os
import subprocess
from typing import Optional

from .. import _lib as L

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "memlayer_xla.cc")
LIB = os.path.join(HERE, "libmemlayer_xla.so")
ROOT = os.path.dirname(os.path.dirname(HERE))
HANDLERS = ("MemlayerPoolForward", "MemlayerLayerForward", "MemlayerLayerBackward")
TARGETS = {"MemlayerPoolForward": "memlayer_pool_forward", "MemlayerLayerForward": "memlayer_layer_forward",
           "MemlayerLayerBackward": "memlayer_layer_backward"}


def jax_available() -> bool:
    try:
        import jax  # noqa: F401
        return hasattr(jax, "ffi")
    except ImportError:
        return False


def build(verbose: bool = False) -> Optional[str]:
    """Compile ``memlayer_xla.cc`` into ``libmemlayer_xla.so`` (linked to
    ``libmemlayer.so``) where JAX is installed; None when it is not."""
    if not jax_available():
        if verbose:
            print("jax_ffi: JAX is not installed; the XLA FFI handlers are not built")
        return None
    import jax
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-o", LIB, SRC, "-I", jax.ffi.include_dir(),
           "-I", os.path.join(ROOT, "include"), "-I", "/usr/local/cuda/include",
           "-L", os.path.dirname(L.LIB_PATH), "-l:libmemlayer.so", "-Wl,-rpath," + os.path.dirname(L.LIB_PATH)]
    subprocess.check_call(cmd)
    return LIB


_registered = False


def register() -> None:
    """Register the handlers as CUDA custom-call targets (once per process)."""
    global _registered
    if _registered:
        return
    if not jax_available():
        raise ImportError("the memory layer's JAX binding needs jax with jax.ffi")
    import jax
    if not os.path.exists(LIB):
        build()
    L.lib()                                         # the kernels' library first (RTLD_GLOBAL not needed)
    h = C.CDLL(LIB)
    for sym in HANDLERS:
        jax.ffi.register_ffi_target(TARGETS[sym], jax.ffi.pycapsule(getattr(h, sym)), platform="CUDA")
    _registered = True


def _attrs(pool) -> dict:
    """MemoryPool fields as the handlers' attributes (memory.py:72-97)."""
    return dict(heads=int(pool.heads), n_sub_keys=int(pool.n_sub_keys), d_key=int(pool.d_key),
                d_value=int(pool.d_value), top_k=int(pool.top_k), routing_noise=float(pool.routing_noise),
                min_temperature=float(pool.min_temperature), max_temperature=float(pool.max_temperature),
                query_scale=int(bool(pool.query_scale)),
                balance_temperature_grad=int(bool(pool.balance_temperature_grad)))


def _empty():
    import jax.numpy as jnp
    return jnp.zeros((0,), jnp.float32)


def pool_forward(pool, queries, sub_keys, log_temperature, values, *, train=False, gumbel=None,
                 noise_scale=1.0, shuffle_reads=False, stats=True):
    """MemoryPool.__call__ through the custom call: (out [..., d], aux), aux
    keyed as memory.py:217-226.  ``pool`` carries the MemoryPool fields;
    ``gumbel`` is the standard Gumbel sample the module draws from its
    "routing" RNG stream when training with noise (memory.py:155-159)."""
    import jax
    import jax.numpy as jnp
    register()
    H, dk, d, k, n = pool.heads, pool.d_key, pool.d_value, pool.top_k, pool.n_sub_keys
    lead = queries.shape[:-2]
    M = math.prod(lead)
    f32 = jnp.float32
    st = lambda *s: jax.ShapeDtypeStruct(s if stats else (0,), f32)  # noqa: E731
    outs = (jax.ShapeDtypeStruct((M, d), f32), jax.ShapeDtypeStruct((M, H, k), jnp.int32),
            jax.ShapeDtypeStruct((M, H, k), f32), jax.ShapeDtypeStruct((1,), f32), jax.ShapeDtypeStruct((1,), f32),
            st(H, 2, n), st(n * n), st(1), st(M, H, 2, dk // 2))
    res = jax.ffi.ffi_call("memlayer_pool_forward", outs)(
        queries.astype(f32), sub_keys.astype(f32), jnp.reshape(log_temperature, (1,)).astype(f32), values,
        _empty() if gumbel is None else gumbel.astype(f32), train=int(bool(train)),
        noise_scale=float(noise_scale), shuffle_reads=int(bool(shuffle_reads)), stats=int(bool(stats)),
        **_attrs(pool))
    out, slots, weights, temp, top1, skc, slc, bal, qu = res
    aux = {"slots": slots.reshape(*lead, H, k), "weights": weights.reshape(*lead, H, k),
           "temperature": temp[0], "top1_weight": top1[0]}
    if stats:
        aux.update(balance_loss=bal[0], subkey_counts=skc, slot_counts=slc, queries=qu)
    return out.reshape(*lead, d), aux


def layer_workspace_bytes(pool, tokens: int, d_model: int, values_dtype: int) -> int:
    cfg = pool.config(tokens, values_dtype, d_model) if hasattr(pool, "config") else None
    if cfg is None:
        raise TypeError("pool must be a model_b200.MemoryPool")
    nb = C.c_size_t()
    L.check(L.lib().memlayer_layer_workspace_size(C.byref(cfg), C.byref(nb)), "memlayer_layer_workspace_size")
    return nb.value


def memory_block(pool, d_model: int, *, train: bool = False, noise_scale: float = 1.0, balance_coef: float = 0.0,
                 route_through_pool: bool = False, shuffle_reads: bool = False):
    """The memory-layer block of model.py:110-119 as a differentiable JAX
    function ``f(h, params, probe, gumbel) -> (y, mem, aux)`` whose backward
    runs ``memlayer_layer_backward``.  ``params`` holds the reference's
    parameters: router / mem_gate / mem_out {kernel, bias}, sub_keys, values,
    log_temperature.  ``probe`` is the zero array [M, d] the reference adds
    to the read (model.py:114-115); its cotangent is the read-output gradient
    that the sparse row update consumes, and the value table itself gets a
    zero gradient (the reference's sparse_grad path).  ``gumbel`` is the
    [M, H, 2, n] selection-noise sample (or an empty array)."""
    import jax
    import jax.numpy as jnp
    register()
    H, dk, d, k, n = pool.heads, pool.d_key, pool.d_value, pool.top_k, pool.n_sub_keys
    f32 = jnp.float32
    dt_code = lambda v: {jnp.dtype(jnp.float16): L.F16, jnp.dtype(jnp.bfloat16): L.BF16}.get(v.dtype, L.F32)  # noqa

    def bias(b):
        return _empty() if b is None else b.astype(f32)

    def fwd_call(h, p, gumbel, noise_scale, train):
        M = h.shape[0]
        ws = layer_workspace_bytes(pool, M, d_model, dt_code(p["values"]))
        outs = (jax.ShapeDtypeStruct((M, d_model), f32), jax.ShapeDtypeStruct((M, d), f32),
                jax.ShapeDtypeStruct((M, H, k), jnp.int32), jax.ShapeDtypeStruct((M, H, k), f32),
                jax.ShapeDtypeStruct((1,), f32), jax.ShapeDtypeStruct((1,), f32),
                jax.ShapeDtypeStruct((H, 2, n), f32), jax.ShapeDtypeStruct((n * n,), f32),
                jax.ShapeDtypeStruct((1,), f32), jax.ShapeDtypeStruct((ws,), jnp.uint8))
        return jax.ffi.ffi_call("memlayer_layer_forward", outs)(
            h.astype(f32), p["router"]["kernel"], bias(p["router"].get("bias")), p["mem_gate"]["kernel"],
            bias(p["mem_gate"].get("bias")), p["mem_out"]["kernel"], bias(p["mem_out"].get("bias")),
            p["sub_keys"], jnp.reshape(p["log_temperature"], (1,)).astype(f32), p["values"],
            _empty() if gumbel is None or gumbel.size == 0 else gumbel.astype(f32), d_model=int(d_model),
            train=int(bool(train)),
            noise_scale=float(noise_scale), shuffle_reads=int(bool(shuffle_reads)), stats=1, **_attrs(pool))

    @jax.custom_vjp
    def block(h, p, probe, gumbel):
        y, mem, slots, weights, temp, top1, skc, slc, bal, _ = fwd_call(h, p, gumbel, noise_scale, train)
        return y, mem, {"slots": slots, "weights": weights, "temperature": temp[0], "top1_weight": top1[0],
                        "subkey_counts": skc, "slot_counts": slc, "balance_loss": bal[0]}

    def block_fwd(h, p, probe, gumbel):
        y, mem, slots, weights, temp, top1, skc, slc, bal, ws = fwd_call(h, p, gumbel, noise_scale, train)
        aux = {"slots": slots, "weights": weights, "temperature": temp[0], "top1_weight": top1[0],
               "subkey_counts": skc, "slot_counts": slc, "balance_loss": bal[0]}
        return (y, mem, aux), (h, p, slots, weights, bal, ws)

    def block_bwd(res, cot):
        h, p, slots, weights, bal, ws = res
        dy = cot[0]
        M = h.shape[0]
        rk, gk, ok_ = p["router"]["kernel"], p["mem_gate"]["kernel"], p["mem_out"]["kernel"]
        outs = tuple(jax.ShapeDtypeStruct(s, f32) for s in (
            (M, d_model), rk.shape, (rk.shape[1],), p["sub_keys"].shape, (1,), gk.shape, (gk.shape[1],),
            ok_.shape, (ok_.shape[1],), (M, d)))
        g = jax.ffi.ffi_call("memlayer_layer_backward", outs)(
            h.astype(f32), rk, bias(p["router"].get("bias")), gk, bias(p["mem_gate"].get("bias")), ok_,
            bias(p["mem_out"].get("bias")), p["sub_keys"], jnp.reshape(p["log_temperature"], (1,)).astype(f32),
            p["values"], slots, weights, bal, ws, dy.astype(f32), d_model=int(d_model),
            shuffle_reads=int(bool(shuffle_reads)), balance_coef=float(balance_coef),
            route_through_pool=int(bool(route_through_pool)), **_attrs(pool))
        dh, dwr, dbr, dsk, dlt, dwg, dbg, dwo, dbo, probe = g
        dp = {"router": {"kernel": dwr, "bias": dbr}, "mem_gate": {"kernel": dwg, "bias": dbg},
              "mem_out": {"kernel": dwo, "bias": dbo}, "sub_keys": dsk,
              "log_temperature": jnp.reshape(dlt, jnp.shape(p["log_temperature"])),
              "values": jnp.zeros_like(p["values"])}
        for name in ("router", "mem_gate", "mem_out"):          # parameters given without a bias
            if p[name].get("bias") is None:
                dp[name].pop("bias")
        return dh, dp, probe, None

    block.defvjp(block_fwd, block_bwd)
    return block
