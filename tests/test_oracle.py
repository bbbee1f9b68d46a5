"""The CPU oracle against the golden fixtures and the reference's own
property tests (restated from tests/test_memory_pool.py of the reference)."""

import numpy as np
import pytest

import inputs as gi
from cases import case_inputs, pool_config, run_oracle
from conftest import golden_names, load_golden
from oracle import memlayer_ref as ref
from parity import OUT_RTOL_F32, OUT_RTOL_HALF, assert_rel, check_slots


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_golden(name):
    recipe, exp = load_golden(name)
    res = run_oracle(recipe)
    aux = res["aux"]
    M, H, k = exp["slots"].shape
    # routing: the golden run used the same float32 operations, so exact
    assert check_slots(res["slots"], exp["slots"], res["route"]["scores"], recipe["n_sub_keys"]) == 0
    np.testing.assert_array_equal(res["slots"], exp["slots"])
    assert_rel(res["weights"], exp["weights"], OUT_RTOL_F32, "weights")
    tol = OUT_RTOL_HALF if recipe.get("values_dtype") else OUT_RTOL_F32
    assert_rel(res["out"], exp["out"], tol, "out")
    if "y" in exp:
        assert_rel(res["y"], exp["y"], OUT_RTOL_F32, "y")
    np.testing.assert_array_equal(aux["subkey_counts"], exp["subkey_counts"])
    assert abs(float(aux["balance_loss"]) - float(exp["balance_loss"])) <= 1e-5 * abs(float(exp["balance_loss"]))
    assert float(aux["temperature"]) == float(exp["temperature"])
    assert abs(float(aux["top1_weight"]) - float(exp["top1_weight"])) <= 1e-6
    if "slot_counts" in exp:
        np.testing.assert_array_equal(aux["slot_counts"], exp["slot_counts"])
        assert_rel(aux["queries"], exp["queries_aux"], 1e-6, "queries")


def test_golden_covers_edge_cases():
    names = set(golden_names())
    for want in ("tiny_ties", "tiny_noise", "tiny_qscale", "tiny_shuffle", "tiny_tlow", "tiny_thigh",
                 "small_k1", "small_kn", "medium_fp16", "medium_bf16", "k32_h8", "cfg0_layer"):
        assert want in names


# ---- properties of the reference suite (tests/test_memory_pool.py) ----
TINY = dict(n_sub_keys=16, heads=2, d_key=8, d_value=12, top_k=4, M=15, seed=7)


def test_shapes_and_weights():
    """test_memory_pool.py:30-37"""
    res = run_oracle(TINY)
    aux = res["aux"]
    assert res["out"].shape == (15, 12) and res["slots"].shape == (15, 2, 4)
    np.testing.assert_allclose(res["weights"].sum(-1), 1.0, rtol=1e-5)
    assert aux["slot_counts"].sum() == 15 * 2 * 4
    np.testing.assert_allclose(aux["subkey_counts"].sum(-1), 15 * 4)


@pytest.mark.parametrize("recipe", [TINY, dict(TINY, n_sub_keys=32, top_k=8, seed=9),
                                    dict(TINY, tie_keys=True, seed=10)])
def test_product_keys_find_exact_top_k(recipe):
    """test_memory_pool.py:40-52: two-stage search == brute force over n^2."""
    res = run_oracle(recipe)
    s = res["route"]["scores"]
    n, k = recipe["n_sub_keys"], recipe["top_k"]
    full = (s[:, :, 0, :, None] + s[:, :, 1, None, :]).reshape(s.shape[0], s.shape[1], n * n)
    _, brute = ref.top_k(full, k)
    np.testing.assert_array_equal(np.sort(res["slots"], -1), np.sort(brute, -1))


def _top_k_by_max(x, k):
    """memory.py:34-45 restated: k rounds of first-argmax + mask-out."""
    x = x.copy()
    vals, idx = [], []
    for _ in range(k):
        i = np.argmax(x, axis=-1)
        vals.append(np.take_along_axis(x, i[..., None], -1)[..., 0])
        idx.append(i)
        np.put_along_axis(x, i[..., None], -np.inf, -1)
    return np.stack(vals, -1), np.stack(idx, -1)


def test_top_k_tie_semantics():
    """test_memory_pool.py:55-63: ties resolve lowest index first."""
    x = gi.hash_normal((64, 100), 3)
    x[:, 10] = x[:, 3]
    x[:, 50] = x[:, 3]
    for k in (1, 4, 16, 100):
        v, i = ref.top_k(x, k)
        v2, i2 = _top_k_by_max(x, k)
        np.testing.assert_array_equal(i, i2)
        np.testing.assert_array_equal(v, v2)


def test_noise_changes_selection_only_in_training():
    """test_memory_pool.py:66-76"""
    r = dict(TINY, noise=5.0, seed=11)
    clean = run_oracle(r)
    noisy = run_oracle(dict(r, train=True))
    off = run_oracle(dict(r, train=True, noise_scale=0.0))
    assert not np.array_equal(clean["slots"], noisy["slots"])
    np.testing.assert_array_equal(clean["slots"], off["slots"])
    # noise only changes which slots are read, never their weights' formula
    s = noisy["route"]["scores"]
    from parity import slot_scores
    w = ref.softmax(slot_scores(s, noisy["slots"], r["n_sub_keys"]))
    np.testing.assert_allclose(noisy["weights"], w, rtol=1e-6)


def test_temperature_clamp():
    """memory.py:141-146 / test_memory_pool.py:79-101 (forward value)."""
    assert abs(float(ref.temperature(np.log(2.0), 5.0, 100.0)) - 5.0) < 1e-4
    assert abs(float(ref.temperature(np.log(500.0), 10.0, 100.0)) - 100.0) < 1e-3
    assert abs(float(ref.temperature(np.log(20.0), 10.0, 100.0)) - 20.0) < 1e-4


def test_query_scale_sharpens_reads_without_changing_picks():
    """test_memory_pool.py:118-125"""
    cfg = pool_config(dict(TINY, query_scale=True))
    x = case_inputs(TINY)
    a_out, a = ref.pool_forward(cfg, x["queries"], x["sub_keys"], x["log_t"], x["values"])
    b_out, b = ref.pool_forward(cfg, x["queries"] * np.float32(10.0), x["sub_keys"], x["log_t"], x["values"])
    np.testing.assert_array_equal(a["slots"], b["slots"])
    assert float(b["top1_weight"]) > float(a["top1_weight"])


def test_balance_loss_detects_collapse():
    """test_memory_pool.py:153-160"""
    cfg = pool_config(TINY)
    x = case_inputs(TINY)
    spread_q = gi.hash_normal((4096, 2, 8), 5)
    collapsed_q = np.broadcast_to(spread_q[:1], spread_q.shape).copy()
    _, spread = ref.pool_forward(cfg, spread_q, x["sub_keys"], x["log_t"], x["values"])
    _, collapsed = ref.pool_forward(cfg, collapsed_q, x["sub_keys"], x["log_t"], x["values"])
    assert spread["balance_loss"] < 1.5
    assert collapsed["balance_loss"] > 2 * spread["balance_loss"]


def test_shuffle_reads_keeps_routing_but_changes_what_is_read():
    """test_memory_pool.py:577-588"""
    base = run_oracle(TINY)
    sh = run_oracle(dict(TINY, shuffle_reads=True))
    np.testing.assert_array_equal(base["slots"], sh["slots"])
    assert not np.allclose(base["out"], sh["out"])
    v = case_inputs(TINY)["values"]
    N = 16 ** 2
    read = (base["slots"] + N // 2 + 1) % N
    manual = np.einsum("mhk,mhkd->md", base["weights"], v[read])
    np.testing.assert_allclose(sh["out"], manual, rtol=1e-5, atol=1e-6)


def test_sparse_row_grads_equal_dense_grads():
    """test_memory_pool.py:321-344 (the value-table part): rows from
    fetched_row_grads scattered into a dense table equal autograd's dense
    gradient of the read, and unfetched rows are exactly zero."""
    torch = pytest.importorskip("torch")
    r = dict(TINY, n_sub_keys=8, M=64, seed=12)
    res = run_oracle(r)
    v = case_inputs(r)["values"]
    g_out = gi.hash_normal(res["out"].shape, 13)
    vt = torch.tensor(v, requires_grad=True)
    rows = vt[torch.tensor(res["slots"])]
    out = torch.einsum("mhk,mhkd->md", torch.tensor(res["weights"]), rows)
    (out * torch.tensor(g_out)).sum().backward()
    dense = vt.grad.numpy()
    uniq, g_rows = ref.fetched_row_grads(res["slots"], res["weights"], g_out, 64)
    scat = np.zeros_like(v)
    scat[uniq] = g_rows
    np.testing.assert_allclose(scat, dense, rtol=1e-4, atol=1e-6)
    untouched = np.setdiff1d(np.arange(64), uniq)
    assert np.all(dense[untouched] == 0)


def test_rowwise_adagrad_changes_only_fetched_rows():
    """test_memory_pool.py:505-513 and train.py:412-416"""
    v = gi.hash_normal((1000, 64), 14)
    acc = np.zeros(1000, np.float32)
    before = v.copy()
    ref.rowwise_adagrad(v, acc, np.array([3, 7]), np.ones((2, 64), np.float32), lr=0.1)
    changed = np.flatnonzero(np.any(v != before, axis=1))
    assert changed.tolist() == [3, 7] and acc[3] == 1.0
    np.testing.assert_allclose(v[3], before[3] - 0.1 / (1.0 + 1e-8), rtol=1e-6)


@pytest.mark.parametrize("name", ["medium", "cfg1_layer_fp16", "tiny_shuffle", "k32_h8"])
def test_oracle_from_slots_reproduces_the_oracle(name):
    """The recomputation used by the GPU tests when a near-tie swapped a
    slot gives the oracle's own outputs and counts from the oracle's own
    selection."""
    from cases import oracle_from_slots, run_oracle
    recipe, _ = load_golden(name)
    orc = run_oracle(recipe)
    fx = oracle_from_slots(recipe, orc["slots"], orc["weights"])
    M = orc["slots"].shape[0]
    np.testing.assert_array_equal(fx["out"].reshape(M, -1), orc["out"].reshape(M, -1))
    np.testing.assert_array_equal(fx["subkey_counts"], orc["aux"]["subkey_counts"])
    np.testing.assert_array_equal(fx["slot_counts"], orc["aux"]["slot_counts"])
    if "y" in orc:
        np.testing.assert_array_equal(fx["y"], orc["y"])
