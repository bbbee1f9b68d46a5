"""Sub-key maintenance on the CPU: the oracle's key_diversity_loss and
revive_dead_keys (memory_pool_model/memory.py:230-281) against restatements
of the reference's own tests (tests/test_memory_pool.py:163-182, 567-574),
the diversity gradient against float64 central differences, and the C ABI's
host-side argument checks (no GPU)."""

import ctypes as C

import numpy as np
import pytest

from model_b200 import _lib as L
from oracle import memlayer_ref as ref


def _unit(x):
    return ref.l2_normalize(np.asarray(x, np.float32))


def test_orthogonal_keys_have_zero_diversity_loss():
    eye = np.eye(4, dtype=np.float32)[None, None]            # reference: test_key_diversity_loss
    loss, grad = ref.key_diversity_loss(eye)
    assert abs(float(loss)) <= 1e-6
    assert np.abs(grad).max() <= 1e-6


def test_identical_keys_have_unit_diversity_loss():
    same = np.ones((1, 1, 4, 4), np.float32)
    loss, _ = ref.key_diversity_loss(same)
    assert float(loss) == pytest.approx(1.0, abs=1e-4)


def test_diversity_loss_matches_pairwise_definition():
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 2, 16, 8)).astype(np.float32)
    loss, _ = ref.key_diversity_loss(x)
    k = x / np.sqrt((x.astype(np.float64) ** 2).sum(-1, keepdims=True) + 1e-6)
    tot = 0.0
    for h in range(2):
        for c in range(2):
            for i in range(16):
                for j in range(16):
                    if i != j:
                        tot += float(k[h, c, i] @ k[h, c, j]) ** 2
    assert float(loss) == pytest.approx(tot / (2 * 2 * 16 * 15), rel=1e-5)


def test_diversity_gradient_matches_central_differences():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((1, 2, 6, 5))

    def f(v):   # float64 restatement of memory.py:236-240
        k = v / np.sqrt((v * v).sum(-1, keepdims=True) + 1e-6)
        g = np.einsum("hcnd,hcmd->hcnm", k, k) * (1 - np.eye(6))
        return (g ** 2).sum() / (1 * 2 * 6 * 5)

    _, grad = ref.key_diversity_loss(x.astype(np.float32))
    num = np.zeros_like(x)
    eps = 1e-6
    for idx in np.ndindex(x.shape):
        p, m = x.copy(), x.copy()
        p[idx] += eps
        m[idx] -= eps
        num[idx] = (f(p) - f(m)) / (2 * eps)
    np.testing.assert_allclose(grad, num, rtol=1e-3, atol=1e-6)


def test_revive_dead_keys_puts_dead_keys_on_queries():
    H, Cb, n, d = 2, 2, 8, 4                                 # reference: test_revive_dead_keys
    rng = np.random.default_rng(0)
    keys = _unit(rng.standard_normal((H, Cb, n, d)))
    usage = np.full((H, Cb, n), 1.0 / n, np.float32)
    usage[0, 1, 3] = 0.0
    usage[1, 0, 5] = 0.0
    queries = _unit(rng.standard_normal((32, H, Cb, d)))
    pick = rng.integers(0, 32, (H, Cb, n))
    noise = rng.standard_normal((H, Cb, n, d)).astype(np.float32)
    new_keys, new_usage, dead = ref.revive_dead_keys(keys, usage, queries, pick, noise, 0.1, noise_scale=0.0)
    assert int(dead.sum()) == 2
    np.testing.assert_array_equal(new_keys[~dead], keys[~dead])
    sims = queries[:, 0, 1] @ new_keys[0, 1, 3]
    assert float(sims.max()) == pytest.approx(1.0, abs=1e-5)
    np.testing.assert_allclose(new_usage, 1.0 / n)


def test_revived_usage_is_still_a_distribution():
    H, Cb, n, d = 2, 2, 8, 4                                 # reference: test_revived_usage_is_still_a_distribution
    rng = np.random.default_rng(1)
    keys = _unit(rng.standard_normal((H, Cb, n, d)))
    usage = rng.dirichlet(np.full(n, 0.3), (H, Cb)).astype(np.float32)
    queries = _unit(rng.standard_normal((32, H, Cb, d)))
    pick = rng.integers(0, 32, (H, Cb, n))
    noise = rng.standard_normal((H, Cb, n, d)).astype(np.float32)
    _, new_usage, dead = ref.revive_dead_keys(keys, usage, queries, pick, noise, 0.5)
    assert int(dead.sum()) > 0
    np.testing.assert_allclose(new_usage.sum(-1), 1.0, rtol=1e-5)


def test_revive_clamps_picks_like_a_gather():
    H, Cb, n, d = 1, 2, 4, 4
    rng = np.random.default_rng(2)
    keys = _unit(rng.standard_normal((H, Cb, n, d)))
    usage = np.zeros((H, Cb, n), np.float32)                 # every key dead
    queries = _unit(rng.standard_normal((5, H, Cb, d)))
    pick = np.array([[[-1, 7, 0, -9], [4, 5, -5, 2]]])
    new_keys, _, _ = ref.revive_dead_keys(keys, usage, queries, pick, np.zeros((H, Cb, n, d), np.float32), 0.1)
    want = np.array([[[4, 4, 0, 0], [4, 4, 0, 2]]])
    for c in range(2):
        for i in range(n):
            np.testing.assert_allclose(new_keys[0, c, i], _unit(queries[want[0, c, i], 0, c]), rtol=1e-6)


def _cfg(H=2, n=8, half=4):
    return L.MemlayerConfig(tokens=0, heads=H, n_sub_keys=n, d_key=2 * half, d_value=4, top_k=1, d_model=0,
                            values_dtype=L.F32, routing_noise=0.0, min_temperature=1.0, max_temperature=1.0)


def test_revive_args_struct_layout():
    assert C.sizeof(L.MemlayerReviveArgs) == 6 * 8 + 2 * 4 + 3 * 8


def test_key_abi_rejects_bad_arguments_on_the_host():
    lib = L.lib()
    cfg = _cfg()
    nb = C.c_size_t()
    assert lib.memlayer_key_diversity_workspace_size(C.byref(cfg), C.byref(nb)) == L.OK
    assert nb.value >= 2 * 2 * 8 * 4 * 4
    assert lib.memlayer_key_diversity_workspace_size(C.byref(cfg), None) == L.ERR_BAD_POINTER
    # neither output
    assert lib.memlayer_key_diversity(C.byref(cfg), 256, None, None, 1.0, 512, nb.value, None) == L.ERR_BAD_POINTER
    # workspace too small / missing
    assert lib.memlayer_key_diversity(C.byref(cfg), 256, 256, None, 1.0, 512, 16, None) == L.ERR_WORKSPACE
    assert lib.memlayer_key_diversity(C.byref(cfg), 256, 256, None, 1.0, None, nb.value, None) == L.ERR_WORKSPACE
    bad = _cfg(H=0)
    assert lib.memlayer_key_diversity(C.byref(bad), 256, 256, None, 1.0, 512, nb.value, None) == L.ERR_BAD_SHAPE
    a = L.MemlayerReviveArgs(sub_keys=256, usage=256, queries=256, query_tokens=0, pick=256, noise=256,
                             threshold=0.1, noise_scale=0.05)
    assert lib.memlayer_revive_dead_keys(C.byref(cfg), C.byref(a), None) == L.ERR_BAD_SHAPE
    a.query_tokens = 4
    a.pick = None
    assert lib.memlayer_revive_dead_keys(C.byref(cfg), C.byref(a), None) == L.ERR_BAD_POINTER
    assert lib.memlayer_revive_dead_keys(C.byref(cfg), None, None) == L.ERR_BAD_POINTER
