"""GPU parity: the CUDA memory layer (through the C ABI) against the golden
fixtures of the reference's memory.py and against the CPU oracle.

Tolerances: slot ids bit-exact except inside near-tie groups (relative gap
<= 1e-6, see parity.check_slots); weights and float32-value outputs within
1e-5 relative; float16/bfloat16-value outputs within 2e-2 relative (max
error over max |ref|; every comparison also bounds the per-element error,
see parity.assert_rel).  Everything downstream of routing (read output,
layer output, sub-key and slot counts) is checked on every call against the
oracle recomputed from the GPU's own slots and weights, so a near-tie swap
never skips a check; without a swap it is also checked against the golden
or oracle outputs directly.
"""

import numpy as np
import pytest
import torch

from cases import case_inputs, oracle_from_slots, pool_config, run_oracle
from conftest import golden_names, load_golden
from oracle import memlayer_ref as ref
from parity import OUT_RTOL_F32, OUT_RTOL_HALF, assert_rel, check_slots

pytestmark = pytest.mark.gpu

DT = {None: torch.float32, "fp16": torch.float16, "bf16": torch.bfloat16}


def _dev(x, dtype=torch.float32):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def run_gpu(recipe, stats=True):
    from model_b200 import MemoryLayer, MemoryPool
    cfg = pool_config(recipe)
    x = case_inputs(recipe)
    pool = MemoryPool(**{f.name: getattr(cfg, f.name) for f in cfg.__dataclass_fields__.values()})
    vdt = DT[recipe.get("values_dtype")]
    params = {"sub_keys": _dev(x["sub_keys"]), "values": _dev(x["values"], vdt),
              "log_temperature": torch.tensor(float(x["log_t"]), device="cuda")}
    kw = dict(train=recipe.get("train", False), noise_scale=recipe.get("noise_scale", 1.0),
              shuffle_reads=recipe.get("shuffle_reads", False), stats=stats, check=True)
    if "gumbel" in x:
        kw["gumbel"] = _dev(x["gumbel"])
    if recipe.get("layer"):
        layer = MemoryLayer(pool, d_model=recipe["d_model"], layer=1)
        lp = {"router_1": {"kernel": _dev(x["w_router"]), "bias": _dev(x["b_router"])},
              "mem_gate_1": {"kernel": _dev(x["w_gate"]), "bias": _dev(x["b_gate"])},
              "mem_out_1": {"kernel": _dev(x["w_out"]), "bias": _dev(x["b_out"])},
              "pool": params}
        y, mem, aux = layer.apply(lp, _dev(x["h"]), **kw)
        res = {"y": y, "out": mem}
    else:
        out, aux = pool.apply({"params": params}, _dev(x["queries"]), **kw)
        res = {"out": out}
    torch.cuda.synchronize()
    res.update(aux)
    return {k: (v.cpu().numpy() if isinstance(v, torch.Tensor) else v) for k, v in res.items()}


@pytest.mark.parametrize("name", golden_names())
def test_gpu_matches_golden_without_stats(name):
    """Inference-style call (no routing statistics): the clean selection
    fast path of the score kernel."""
    recipe, exp = load_golden(name)
    got = run_gpu(recipe, stats=False)
    orc = run_oracle(recipe)
    M, H, k = exp["slots"].shape
    swapped = check_slots(got["slots"], exp["slots"], orc["route"]["scores"], recipe["n_sub_keys"])
    tol = OUT_RTOL_HALF if recipe.get("values_dtype") else OUT_RTOL_F32
    x = case_inputs(recipe)
    mix = ref.gather_mix(x["values"], got["slots"].reshape(M, H, k).astype(np.int64), got["weights"].reshape(M, H, k),
                         recipe.get("shuffle_reads", False))
    assert_rel(got["out"].reshape(M, -1), mix, tol, "out vs oracle mix of chosen slots")
    fx = oracle_from_slots(recipe, got["slots"], got["weights"])
    if "y" in exp:
        assert_rel(got["y"], fx["y"], OUT_RTOL_F32, "y vs oracle from the GPU's slots")
    if swapped == 0:
        assert_rel(got["out"], exp["out"], tol, "out vs golden")
        if "y" in exp:
            assert_rel(got["y"], exp["y"], OUT_RTOL_F32, "y vs golden")


@pytest.mark.parametrize("name", golden_names())
def test_gpu_matches_golden(name):
    recipe, exp = load_golden(name)
    got = run_gpu(recipe)
    orc = run_oracle(recipe)
    n = recipe["n_sub_keys"]
    swapped = check_slots(got["slots"], exp["slots"], orc["route"]["scores"], n)
    tol = OUT_RTOL_HALF if recipe.get("values_dtype") else OUT_RTOL_F32
    # weights are the softmax of the oracle scores at the slots the GPU chose
    from parity import slot_scores
    M, H, k = exp["slots"].shape
    w_ref = ref.softmax(slot_scores(orc["route"]["scores"], got["slots"].reshape(M, H, k).astype(np.int64), n))
    assert_rel(got["weights"].reshape(M, H, k), w_ref, OUT_RTOL_F32, "weights")
    x = case_inputs(recipe)
    fx = oracle_from_slots(recipe, got["slots"], got["weights"])
    np.testing.assert_array_equal(got["subkey_counts"], fx["subkey_counts"])
    if "slot_counts" in got:
        np.testing.assert_array_equal(got["slot_counts"], fx["slot_counts"])
    if "y" in exp:
        assert_rel(got["y"], fx["y"], OUT_RTOL_F32, "y vs oracle from the GPU's slots")
    if swapped == 0:
        np.testing.assert_array_equal(got["slots"].astype(np.int64), exp["slots"])
        assert_rel(got["weights"], exp["weights"], OUT_RTOL_F32, "weights vs golden")
        assert_rel(got["out"], exp["out"], tol, "out vs golden")
        if "y" in exp:
            assert_rel(got["y"], exp["y"], OUT_RTOL_F32, "y vs golden")
        np.testing.assert_array_equal(got["subkey_counts"], exp["subkey_counts"])
        if "slot_counts" in exp:
            np.testing.assert_array_equal(got["slot_counts"], exp["slot_counts"])
    # output of the chosen slots, mixed by the oracle
    mix = ref.gather_mix(x["values"], got["slots"].reshape(M, H, k).astype(np.int64), got["weights"].reshape(M, H, k),
                         recipe.get("shuffle_reads", False))
    assert_rel(got["out"].reshape(M, -1), mix, tol, "out vs oracle mix of chosen slots")
    assert abs(float(got["balance_loss"]) - float(exp["balance_loss"])) <= 1e-5 * abs(float(exp["balance_loss"])) + 1e-6
    assert abs(float(got["temperature"]) - float(exp["temperature"])) <= 1e-6 * float(exp["temperature"])
    assert abs(float(got["top1_weight"]) - float(exp["top1_weight"])) <= 1e-5
    if "queries_aux" in exp:
        assert_rel(got["queries"], exp["queries_aux"], 1e-6, "queries")


def test_gpu_noise_anneal_and_eval_are_clean():
    """test_memory_pool.py:66-76 on the CUDA path."""
    r = dict(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4, M=15, seed=21, noise=5.0)
    clean = run_gpu(r)
    noisy = run_gpu(dict(r, train=True))
    off = run_gpu(dict(r, train=True, noise_scale=0.0))
    assert not np.array_equal(clean["slots"], noisy["slots"])
    np.testing.assert_array_equal(clean["slots"], off["slots"])


def test_gpu_empty_input():
    from model_b200 import MemoryPool
    pool = MemoryPool(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4)
    params = pool.init(0)
    out, aux = pool.apply(params, torch.zeros(0, 2, 8, device="cuda"))
    torch.cuda.synchronize()
    assert out.shape == (0, 12) and aux["slots"].shape == (0, 2, 4)
    assert float(aux["slot_counts"].sum()) == 0.0


def test_gpu_leading_dims_and_query_scale_keeps_picks():
    """test_memory_pool.py:118-125 with [3, 5, H, d_key] queries."""
    from model_b200 import MemoryPool
    pool = MemoryPool(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4, query_scale=True)
    params = pool.init(1)
    q = torch.randn(3, 5, 2, 8, device="cuda", generator=torch.Generator("cuda").manual_seed(0))
    out_a, a = pool.apply(params, q)
    out_b, b = pool.apply(params, q * 10.0)
    assert out_a.shape == (3, 5, 12) and a["slots"].shape == (3, 5, 2, 4)
    assert torch.equal(a["slots"], b["slots"])
    assert float(b["top1_weight"]) > float(a["top1_weight"])


@pytest.mark.parametrize("values_dtype", ["f32", "bf16", "f32_nostats"])
def test_gpu_full_config0_against_oracle(values_dtype):
    """configs[0] at full size (T=8192, n=512, H=4, k=16, d=256): routing and
    outputs against the oracle on the same seeded inputs."""
    recipe = dict(n_sub_keys=512, heads=4, d_key=256, d_value=256, top_k=16, M=8192, seed=0, layer=True,
                  d_model=256, key_std=float(np.sqrt(1 / 128)))
    if values_dtype == "bf16":
        recipe["values_dtype"] = "bf16"
    stats = values_dtype != "f32_nostats"
    got = run_gpu(recipe, stats=stats)
    orc = run_oracle(recipe)
    M, H, k = orc["slots"].shape
    swapped = check_slots(got["slots"], orc["slots"], orc["route"]["scores"], 512)
    assert swapped <= M * H // 1000, swapped
    x = case_inputs(recipe)
    mix = ref.gather_mix(x["values"], got["slots"].astype(np.int64), got["weights"])
    tol = OUT_RTOL_HALF if values_dtype == "bf16" else OUT_RTOL_F32
    assert_rel(got["out"], mix, tol, "out")
    fx = oracle_from_slots(recipe, got["slots"], got["weights"])
    assert_rel(got["y"], fx["y"], OUT_RTOL_F32, "y vs oracle from the GPU's slots")
    if stats:
        np.testing.assert_array_equal(got["subkey_counts"], fx["subkey_counts"])
        np.testing.assert_array_equal(got["slot_counts"], fx["slot_counts"])
    if swapped == 0:
        assert_rel(got["y"], orc["y"], OUT_RTOL_F32, "y")
        if stats:
            np.testing.assert_array_equal(got["subkey_counts"], orc["aux"]["subkey_counts"])
    np.testing.assert_allclose(got["weights"].sum(-1), 1.0, rtol=1e-5)
    if stats:
        assert got["slot_counts"].sum() == M * H * k
        assert abs(float(got["balance_loss"]) - float(orc["aux"]["balance_loss"])) <= \
            1e-5 * float(orc["aux"]["balance_loss"])


SHAPES = {
    # n not a multiple of the 256-key chunk, ragged token count
    "n300_m200": dict(n_sub_keys=300, heads=2, d_key=64, d_value=32, top_k=16, M=200, seed=31),
    "cfg0_m1000": dict(n_sub_keys=512, heads=4, d_key=256, d_value=256, top_k=16, M=1000, seed=32,
                       key_std=float(np.sqrt(1 / 128))),
    # billion-slot config's head / top-k shape at a small n
    "k32_h8_n1024": dict(n_sub_keys=1024, heads=8, d_key=256, d_value=64, top_k=32, M=300, seed=33),
    "qscale_m129": dict(n_sub_keys=256, heads=4, d_key=128, d_value=256, top_k=16, M=129, seed=34, query_scale=True),
    "noise_train": dict(n_sub_keys=512, heads=4, d_key=128, d_value=64, top_k=16, M=256, seed=35, noise=1.0,
                        train=True, noise_scale=0.5),
    "btgrad_bf16": dict(n_sub_keys=128, heads=4, d_key=64, d_value=128, top_k=8, M=512, seed=36, query_scale=True,
                        balance_temperature_grad=True, values_dtype="bf16"),
    "k4_n64": dict(n_sub_keys=64, heads=1, d_key=64, d_value=16, top_k=4, M=130, seed=37),
    # layer block with tensor-core projections (M >= 128), biases on, ragged M
    "layer_cfg1_m300": dict(n_sub_keys=512, heads=4, d_key=128, d_value=256, top_k=16, M=300, seed=38, layer=True,
                            d_model=256, biases=True, values_dtype="fp16"),
    "layer_h8_m257": dict(n_sub_keys=256, heads=8, d_key=64, d_value=64, top_k=32, M=257, seed=39, layer=True,
                          d_model=96, biases=True),
    "layer_qscale_noise": dict(n_sub_keys=128, heads=2, d_key=256, d_value=128, top_k=8, M=384, seed=40, layer=True,
                               d_model=128, query_scale=True, noise=1.0, train=True, clustered=True),
    # router 128 + gate 64 columns (< one 256-column tile): the float32 SIMT projections
    "layer_n192": dict(n_sub_keys=128, heads=2, d_key=64, d_value=64, top_k=8, M=300, seed=41, layer=True,
                       d_model=64, biases=True),
    "layer_n192_qscale_noise": dict(n_sub_keys=128, heads=2, d_key=64, d_value=64, top_k=8, M=300, seed=42,
                                    layer=True, d_model=64, query_scale=True, noise=1.0, train=True),
}


@pytest.mark.parametrize("stats", [True, False])
@pytest.mark.parametrize("name", sorted(SHAPES))
def test_gpu_shapes_against_oracle(name, stats):
    """Tensor-core score path at edge shapes: routing, weights, outputs and
    the balance loss against the oracle on the same inputs (stats=False
    takes the clean-selection fast path)."""
    recipe = SHAPES[name]
    got = run_gpu(recipe, stats=stats)
    orc = run_oracle(recipe)
    n = recipe["n_sub_keys"]
    M, H, k = orc["slots"].shape
    swapped = check_slots(got["slots"], orc["slots"], orc["route"]["scores"], n)
    assert swapped <= max(1, M * H // 500), swapped
    from parity import slot_scores
    w_ref = ref.softmax(slot_scores(orc["route"]["scores"], got["slots"].reshape(M, H, k).astype(np.int64), n))
    assert_rel(got["weights"].reshape(M, H, k), w_ref, OUT_RTOL_F32, "weights")
    x = case_inputs(recipe)
    tol = OUT_RTOL_HALF if recipe.get("values_dtype") else OUT_RTOL_F32
    mix = ref.gather_mix(x["values"], got["slots"].reshape(M, H, k).astype(np.int64), got["weights"].reshape(M, H, k))
    assert_rel(got["out"].reshape(M, -1), mix, tol, "out")
    if stats:
        assert abs(float(got["balance_loss"]) - float(orc["aux"]["balance_loss"])) <= \
            1e-5 * float(orc["aux"]["balance_loss"])
    fx = oracle_from_slots(recipe, got["slots"], got["weights"])
    if stats:
        np.testing.assert_array_equal(got["subkey_counts"], fx["subkey_counts"])
        np.testing.assert_array_equal(got["slot_counts"], fx["slot_counts"])
    if "y" in fx:
        assert_rel(got["y"], fx["y"], tol if recipe.get("values_dtype") else OUT_RTOL_F32,
                   "y vs oracle from the GPU's slots")
    if swapped == 0:
        if stats:
            np.testing.assert_array_equal(got["subkey_counts"], orc["aux"]["subkey_counts"])
        if "y" in orc:
            assert_rel(got["y"], orc["y"], tol if recipe.get("values_dtype") else OUT_RTOL_F32, "y")
    if recipe.get("layer") and stats:
        assert_rel(got["queries"].reshape(M, H, 2, -1), orc["route"]["q"], 1e-5, "unit queries")


@pytest.mark.parametrize("M,chunks", [(8192, 4), (3000, 3), (1000, 8), (200, 4)])
def test_gpu_layer_forward_host_buffers(M, chunks):
    """memlayer_layer_forward_host (host h / y, chunked copy-compute
    pipeline) gives the device entry's results bit for bit."""
    from model_b200 import MemoryLayer, MemoryPool
    pool = MemoryPool(n_sub_keys=128, heads=4, d_key=128, d_value=128, top_k=16)
    layer = MemoryLayer(pool, d_model=128, layer=1)
    params = layer.init(4)
    h = torch.randn(M, 128, generator=torch.Generator().manual_seed(M))
    y_dev, _, aux_dev = layer.apply(params, h.cuda(), check=True)
    for _ in range(2):                 # the workspace / staging buffers are reused across calls
        y_host, aux = layer.apply_host(params, h, chunks=chunks, check=True)
    torch.cuda.synchronize()
    assert torch.equal(aux["slots"], aux_dev["slots"])
    assert torch.equal(aux["weights"], aux_dev["weights"])
    assert torch.equal(y_host, y_dev.cpu())


def _big_pool_case(n, H, dk, d, k, vdt, M, seed):
    """Routing of the large configs against the oracle; the read against a
    torch gather of the same table with the kernel's own slots and weights."""
    from model_b200 import MemoryPool
    pool = MemoryPool(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k)
    g = torch.Generator("cuda").manual_seed(seed)
    sk = torch.randn(H, 2, n, dk // 2, device="cuda", generator=g)
    values = torch.randn(n * n, d, device="cuda", generator=g, dtype=vdt).mul_(0.02)   # no float32 copy
    params = {"sub_keys": sk, "values": values,
              "log_temperature": torch.tensor(np.log(10.0), device="cuda", dtype=torch.float32)}
    q = torch.randn(M, H, dk, device="cuda", generator=g)
    out, aux = pool.apply({"params": params}, q, stats=False, check=True)
    torch.cuda.synchronize()
    cfg = ref.PoolConfig(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k)
    r = ref.route(cfg, q.cpu().numpy(), sk.cpu().numpy(), float(np.log(10.0)))
    check_slots(aux["slots"].cpu().numpy(), r["slots"], r["scores"], n)
    w_ref = ref.softmax(r["slot_scores"])
    same = (aux["slots"].cpu().numpy() == r["slots"]).all(-1)
    np.testing.assert_allclose(aux["weights"].cpu().numpy()[same], w_ref[same], rtol=1e-5, atol=1e-7)
    rows = values[aux["slots"].long()].float()                       # [M, H, k, d]
    want = torch.einsum("mhk,mhkd->md", aux["weights"], rows)
    assert_rel(out.cpu().numpy(), want.cpu().numpy(), 1e-5, "read")
    del values, rows
    torch.cuda.empty_cache()


def test_gpu_cfg2_pool_shapes_decode_batches():
    """n_sub_keys 8192 (67,108,864 slots), H 4, d_key 128, top_k 16,
    fp16 rows (d reduced to 64 to bound the test's memory), decode batches."""
    for M in (1, 8, 64):
        _big_pool_case(8192, 4, 128, 64, 16, torch.float16, M, seed=M)


def test_gpu_cfg3_pool_shapes():
    """configs[3] routing: n_sub_keys 32768 (2^30 slots), H 8, d_key 256,
    top_k 32, bf16 rows (d reduced to 16: a 34 GB table on one GPU)."""
    _big_pool_case(32768, 8, 256, 16, 32, torch.bfloat16, 48, seed=3)


@pytest.mark.parametrize("M,n,k,qscale,noisy", [(1, 300, 16, False, False), (7, 300, 8, True, False),
                                                 (33, 1000, 32, False, True), (64, 2048, 16, True, True),
                                                 (64, 256, 4, False, False)])
def test_gpu_few_token_score_path(M, n, k, qscale, noisy):
    """Decode-size calls (M <= 64, no routing statistics) take the split-key
    score path: slots, weights and the read against the oracle, with ragged
    last slices, query_scale and selection noise."""
    from model_b200 import MemoryPool
    H, dk, d = 2, 64, 32
    pool = MemoryPool(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k, query_scale=qscale,
                      routing_noise=2.0 if noisy else 0.0)
    rng = np.random.default_rng(M * 1000 + n)
    sk = rng.standard_normal((H, 2, n, dk // 2)).astype(np.float32)
    values = (rng.standard_normal((n * n, d)) * 0.02).astype(np.float32)
    q = rng.standard_normal((M, H, dk)).astype(np.float32)
    gum = rng.gumbel(size=(M, H, 2, n)).astype(np.float32) if noisy else None
    params = {"sub_keys": _dev(sk), "values": _dev(values),
              "log_temperature": torch.tensor(np.log(10.0), dtype=torch.float32, device="cuda")}
    kw = dict(train=noisy, stats=False, check=True)
    if noisy:
        kw["gumbel"] = _dev(gum)
    out, aux = pool.apply({"params": params}, _dev(q), **kw)
    torch.cuda.synchronize()
    cfg = ref.PoolConfig(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k, query_scale=qscale,
                         routing_noise=2.0 if noisy else 0.0)
    o_ref, a_ref = ref.pool_forward(cfg, q, sk, float(np.log(10.0)), values, train=noisy, gumbel=gum,
                                    with_stats=False)
    r = ref.route(cfg, q, sk, float(np.log(10.0)), noisy, gum)
    check_slots(aux["slots"].cpu().numpy(), a_ref["slots"], r["select"], n)
    same = (aux["slots"].cpu().numpy() == a_ref["slots"]).all(-1)
    np.testing.assert_allclose(aux["weights"].cpu().numpy()[same], a_ref["weights"][same], rtol=1e-5, atol=1e-7)
    if same.all():
        assert_rel(out.cpu().numpy(), o_ref, OUT_RTOL_F32, "out")


@pytest.mark.parametrize("half,k,stats", [(32, 8, False), (32, 8, True), (64, 8, True), (32, 16, True)])
def test_gpu_tensor_core_noisy_selection_narrow_halves(half, k, stats):
    """Selection noise on the tensor-core score path (>= 128 tokens) with
    narrow query halves: slots, weights and the read against the oracle."""
    from model_b200 import MemoryPool
    M, H, n, d = 300, 2, 128, 32
    dk = 2 * half
    pool = MemoryPool(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k, query_scale=True, routing_noise=1.0)
    rng = np.random.default_rng(half * 100 + k)
    sk = rng.standard_normal((H, 2, n, half)).astype(np.float32)
    values = (rng.standard_normal((n * n, d)) * 0.02).astype(np.float32)
    q = rng.standard_normal((M, H, dk)).astype(np.float32)
    gum = rng.gumbel(size=(M, H, 2, n)).astype(np.float32)
    params = {"sub_keys": _dev(sk), "values": _dev(values),
              "log_temperature": torch.tensor(np.log(10.0), dtype=torch.float32, device="cuda")}
    out, aux = pool.apply({"params": params}, _dev(q), train=True, stats=stats, check=True, gumbel=_dev(gum))
    torch.cuda.synchronize()
    cfg = ref.PoolConfig(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k, query_scale=True, routing_noise=1.0)
    o_ref, a_ref = ref.pool_forward(cfg, q, sk, float(np.log(10.0)), values, train=True, gumbel=gum,
                                    with_stats=False)
    r = ref.route(cfg, q, sk, float(np.log(10.0)), True, gum)
    check_slots(aux["slots"].cpu().numpy(), a_ref["slots"], r["select"], n)
