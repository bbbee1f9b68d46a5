"""Generate the golden fixtures by running the reference's own memory layer.

The reference (KumarDev7/model) is pure JAX/Flax, and JAX is not installed
in this environment.  This script imports the reference's
``memory_pool_model/memory.py`` *source file unchanged* on top of
``jaxshim`` (a numpy stand-in for the JAX/Flax primitives that file calls)
and records what ``MemoryPool.apply`` returns for a set of seeded cases.
The Dense/SiLU steps of ``model.py:110-119`` around the pool are plain
``x @ W + b`` / ``x * sigmoid(x)``, applied here in numpy.

Usage (needs the reference checkout; writes tests/golden/*.npz):

    python tests/golden/make_golden.py [/path/to/reference]

Every input is regenerated from the recipe stored in each fixture
(``inputs.pool_inputs``), so the fixtures hold only recipes and outputs.
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import inputs as gi  # noqa: E402
import jaxshim  # noqa: E402

F32 = np.float32

CASES = {
    # the reference tests' make_pool shapes (tests/test_memory_pool.py:19-27)
    "tiny": dict(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4, M=15, seed=100),
    "tiny_ties": dict(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4, M=15, seed=101, tie_keys=True),
    "tiny_qscale": dict(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4, M=15, seed=102, query_scale=True),
    "tiny_noise": dict(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4, M=15, seed=103, train=True,
                       noise=5.0, noise_scale=0.7),
    "tiny_shuffle": dict(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4, M=15, seed=104, shuffle_reads=True),
    "tiny_tlow": dict(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4, M=15, seed=105,
                      log_t=float(np.log(F32(2.0))), min_temperature=5.0),
    "tiny_thigh": dict(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4, M=15, seed=106,
                       log_t=float(np.log(F32(500.0)))),
    "tiny_btgrad": dict(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4, M=15, seed=107,
                        query_scale=True, balance_temperature_grad=True),
    "small_k1": dict(n_sub_keys=8, heads=1, d_key=4, d_value=8, top_k=1, M=9, seed=108),
    "small_kn": dict(n_sub_keys=8, heads=3, d_key=6, d_value=8, top_k=8, M=9, seed=109),
    "medium": dict(n_sub_keys=64, heads=4, d_key=32, d_value=64, top_k=8, M=256, seed=110),
    "medium_ties": dict(n_sub_keys=64, heads=4, d_key=32, d_value=64, top_k=8, M=256, seed=111, tie_keys=True),
    "medium_fp16": dict(n_sub_keys=64, heads=4, d_key=32, d_value=64, top_k=8, M=256, seed=112,
                        values_dtype="fp16"),
    "medium_bf16": dict(n_sub_keys=64, heads=4, d_key=32, d_value=64, top_k=8, M=256, seed=113,
                        values_dtype="bf16"),
    "k32_h8": dict(n_sub_keys=128, heads=8, d_key=64, d_value=32, top_k=32, M=64, seed=114),
    # a slice of the single-layer benchmark shapes: router + pool + gate + out
    "cfg0_layer": dict(n_sub_keys=512, heads=4, d_key=256, d_value=256, top_k=16, M=64, seed=0,
                       layer=True, d_model=256, key_std=float(np.sqrt(1 / 128))),
    "cfg1_layer_fp16": dict(n_sub_keys=512, heads=4, d_key=128, d_value=256, top_k=16, M=64, seed=1,
                            layer=True, d_model=256, values_dtype="fp16", biases=True),
    "cfg4_layer_clustered": dict(n_sub_keys=512, heads=4, d_key=256, d_value=256, top_k=16, M=64, seed=4,
                                 layer=True, d_model=256, clustered=True,
                                 key_std=float(np.sqrt(1 / 128))),
}

POOL_FIELDS = ("n_sub_keys", "heads", "d_key", "d_value", "top_k", "routing_noise", "init_temperature",
               "min_temperature", "balance_temperature_grad", "max_temperature", "query_scale")


def load_reference_memory(ref_root: str):
    jaxshim.install()
    path = os.path.join(ref_root, "memory_pool_model", "memory.py")
    spec = importlib.util.spec_from_file_location("ref_memory", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules["ref_memory"] = mod
    spec.loader.exec_module(mod)
    return mod


def pool_kwargs(recipe: dict) -> dict:
    kw = {k: recipe[k] for k in ("n_sub_keys", "heads", "d_key", "d_value", "top_k")}
    kw["routing_noise"] = recipe.get("noise", 0.0)
    for k in ("min_temperature", "max_temperature", "balance_temperature_grad", "query_scale"):
        if k in recipe:
            kw[k] = recipe[k]
    return kw


def run_case(mem, name: str, recipe: dict, backend: str) -> dict:
    jaxshim.set_backend(backend)
    x = gi.pool_inputs(recipe)
    pool = mem.MemoryPool(**pool_kwargs(recipe))
    params = {"params": {"sub_keys": x["sub_keys"], "values": x["values"],
                         "log_temperature": np.asarray(x["log_t"], F32)}}
    res = {}
    if recipe.get("layer"):
        M = recipe["M"]
        q = (x["h"] @ x["w_router"] + x["b_router"]).astype(F32)                  # model.py:110
        q = q.reshape(M, recipe["heads"], recipe["d_key"])                         # model.py:111
    else:
        q = x["queries"]
    jaxshim.set_gumbel(x.get("gumbel"))
    out, aux = pool.apply(params, q, train=recipe.get("train", False),
                          noise_scale=recipe.get("noise_scale", 1.0),
                          shuffle_reads=recipe.get("shuffle_reads", False))
    res["out"] = np.asarray(out, F32)
    if recipe.get("layer"):
        g = (x["h"] @ x["w_gate"] + x["b_gate"]).astype(F32)
        gate = (g / (F32(1.0) + np.exp(-g))).astype(F32)                           # model.py:118
        res["y"] = ((res["out"] * gate).astype(F32) @ x["w_out"] + x["b_out"]).astype(F32)  # model.py:119
    for key in ("slots", "weights", "subkey_counts", "balance_loss", "temperature", "top1_weight"):
        res[key] = np.asarray(aux[key])
    res["slots"] = res["slots"].astype(np.int64)
    if recipe["n_sub_keys"] ** 2 <= 65536:
        res["slot_counts"] = np.asarray(aux["slot_counts"], F32)
        res["queries_aux"] = np.asarray(aux["queries"], F32)
    return res


def main(ref_root: str) -> None:
    mem = load_reference_memory(ref_root)
    for name, recipe in CASES.items():
        res = run_case(mem, name, recipe, "gpu")
        # memory.py picks its top-k helper by backend: both must agree
        if recipe["top_k"] <= 32:
            alt = run_case(mem, name, recipe, "cpu")
            for key in ("slots", "weights", "out"):
                assert np.array_equal(res[key], alt[key]), (name, key)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), recipe=json.dumps(recipe), **res)
        print(f"{name}: slots {res['slots'].shape} out {res['out'].shape}")


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (the KumarDev7/model checkout)")
    main(root)
