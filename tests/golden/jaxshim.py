"""A numpy stand-in for the few JAX / Flax primitives that the reference's
``memory_pool_model/memory.py`` calls, so that file's own source can run in
this environment (JAX is not installed here) and produce golden vectors.

Only what ``MemoryPool.setup`` / ``MemoryPool.__call__`` (memory.py:94-227)
touch is provided.  Semantics follow JAX's documentation:

* float32 everywhere (Python scalars are weakly typed, as in JAX);
* ``jnp.argmax`` returns the first maximal index;
* ``lax.top_k`` returns values descending, equal values lowest index first;
* ``jax.nn.softmax`` is exp(x - max) / sum(exp(x - max));
* ``x.at[i].add(v)`` is an out-of-place scatter-add;
* ``stop_gradient`` / ``optimization_barrier`` are the identity in a forward pass.

This is test infrastructure used only by ``make_golden.py``; it never ships.
"""

from __future__ import annotations

import dataclasses
import sys
import types

import numpy as np

F32 = np.float32


class JArr(np.ndarray):
    """ndarray with JAX's functional ``.at[idx].add(v)``."""

    @property
    def at(self):
        arr = self

        class _Idx:
            def __getitem__(self, idx):
                class _Op:
                    def add(self, v):
                        out = np.array(arr, copy=True)
                        np.add.at(out, idx, v)
                        return out.view(JArr)
                return _Op()
        return _Idx()


def _f(x):
    """Python scalars -> float32 (JAX weak typing); arrays unchanged."""
    if isinstance(x, (bool, int, float)):
        return F32(x)
    return x


def _make_jnp():
    jnp = types.ModuleType("jax.numpy")
    jnp.float32 = F32
    jnp.int32 = np.int32
    jnp.inf = np.inf
    jnp.ndarray = np.ndarray
    jnp.sum = lambda x, axis=None, keepdims=False: np.sum(x, axis=axis, keepdims=keepdims,
                                                         dtype=x.dtype if x.dtype.kind == "f" else None)
    jnp.mean = lambda x, axis=None, keepdims=False: np.mean(x, axis=axis, keepdims=keepdims)
    jnp.sqrt = lambda x: np.sqrt(_f(x))
    jnp.log = lambda x: np.log(_f(x))
    jnp.exp = lambda x: np.exp(_f(x))
    jnp.clip = lambda x, lo, hi: np.clip(x, lo, hi).astype(np.result_type(x, F32))
    jnp.asarray = lambda x, dtype=None: np.asarray(x, dtype if dtype is not None else F32)
    jnp.arange = np.arange
    jnp.where = np.where
    jnp.stack = np.stack
    jnp.argmax = lambda x, axis=None: np.argmax(x, axis=axis)
    jnp.take_along_axis = np.take_along_axis
    jnp.take = lambda a, idx, axis=None: np.take(a, idx, axis=axis)
    jnp.einsum = lambda spec, *ops: np.einsum(spec, *ops).astype(F32)
    jnp.eye = lambda n, dtype=F32: np.eye(n, dtype=dtype)
    jnp.zeros = lambda shape, dtype=F32: np.zeros(shape, dtype).view(JArr)
    return jnp


def _top_k(x, k):
    n = x.shape[-1]
    flat = x.reshape(-1, n)
    # stable argsort of the negated values: descending, ties lowest index first
    idx = np.argsort(-flat, axis=-1, kind="stable")[:, :k]
    vals = np.take_along_axis(flat, idx, axis=-1)
    return vals.reshape(*x.shape[:-1], k), idx.reshape(*x.shape[:-1], k)


class _State:
    backend = "gpu"          # "gpu" exercises memory.py's own _top_k_by_max
    gumbel = None            # the standard Gumbel sample to hand out


def _make_jax():
    jax = types.ModuleType("jax")
    jax.numpy = _make_jnp()
    jax.Array = np.ndarray
    lax = types.ModuleType("jax.lax")
    lax.rsqrt = lambda x: F32(1.0) / np.sqrt(x)
    lax.stop_gradient = lambda x: x
    lax.optimization_barrier = lambda x: x
    lax.top_k = _top_k
    jax.lax = lax
    nn = types.ModuleType("jax.nn")

    def softmax(x, axis=-1):
        e = np.exp(x - np.max(x, axis=axis, keepdims=True))
        return e / np.sum(e, axis=axis, keepdims=True, dtype=x.dtype)
    nn.softmax = softmax
    jax.nn = nn
    rnd = types.ModuleType("jax.random")

    def gumbel(key, shape):
        g = _State.gumbel
        assert g is not None and tuple(g.shape) == tuple(shape), "set jaxshim.set_gumbel first"
        return g
    rnd.gumbel = gumbel
    rnd.normal = lambda key, shape, dtype=F32: (_ for _ in ()).throw(
        RuntimeError("init is not supported; pass parameters explicitly"))
    rnd.split = lambda key, n=2: [key] * n
    jax.random = rnd
    jax.default_backend = lambda: _State.backend
    return jax


def _make_flax():
    flax = types.ModuleType("flax")
    linen = types.ModuleType("flax.linen")

    class Module:
        def __init_subclass__(cls, **kw):
            super().__init_subclass__(**kw)
            dataclasses.dataclass(cls)

        def apply(self, variables, *args, rngs=None, **kwargs):
            bound = dataclasses.replace(self)
            object.__setattr__(bound, "_params", variables["params"])
            bound.setup()
            return bound(*args, **kwargs)

        def param(self, name, init_fn, *args):
            return self._params[name]

        def make_rng(self, name):
            return name

    class _Init:
        @staticmethod
        def normal(stddev=1.0):
            return lambda key, shape, dtype=F32: None
    linen.Module = Module
    linen.initializers = _Init
    linen.silu = lambda x: x / (F32(1.0) + np.exp(-x))
    flax.linen = linen
    return flax, linen


def install() -> None:
    """Register the stand-ins as ``jax`` / ``flax`` in sys.modules."""
    jax = _make_jax()
    flax, linen = _make_flax()
    sys.modules.update({"jax": jax, "jax.numpy": jax.numpy, "jax.lax": jax.lax,
                        "jax.nn": jax.nn, "jax.random": jax.random,
                        "flax": flax, "flax.linen": linen})


def set_backend(name: str) -> None:
    _State.backend = name


def set_gumbel(g) -> None:
    _State.gumbel = None if g is None else np.asarray(g, F32)
