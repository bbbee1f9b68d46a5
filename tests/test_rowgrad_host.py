"""Row-gradient / Adagrad entry points: argument checks and workspace sizes
on the host (no CUDA call is reached), and the oracle's multi-read merge
against a dense scatter."""

import ctypes as C

import numpy as np

from model_b200 import _lib as L
from oracle import memlayer_ref as ref


def _cfg(**kw):
    base = dict(tokens=0, heads=4, n_sub_keys=64, d_key=2, d_value=64, top_k=16, d_model=0, values_dtype=L.F32,
                routing_noise=0.0, min_temperature=1.0, max_temperature=1.0)
    base.update(kw)
    return L.MemlayerConfig(**base)


def test_rowgrad_workspace_grows_with_fetches():
    lib = L.lib()
    a, b = C.c_size_t(), C.c_size_t()
    assert lib.memlayer_rowgrad_workspace_size(C.byref(_cfg()), 1000, C.byref(a)) == L.OK
    assert lib.memlayer_rowgrad_workspace_size(C.byref(_cfg()), 100000, C.byref(b)) == L.OK
    assert b.value > a.value
    assert lib.memlayer_rowgrad_workspace_size(C.byref(_cfg()), 1 << 31, C.byref(b)) == L.ERR_BAD_SHAPE
    assert lib.memlayer_rowgrad_workspace_size(C.byref(_cfg()), -1, C.byref(b)) == L.ERR_BAD_SHAPE


def test_rowgrad_arguments_rejected_on_the_host():
    lib = L.lib()
    cfg = _cfg()
    fake = 4096                                      # never dereferenced: every call fails its checks first
    rd = L.MemlayerRead(slots=fake, weights=fake, grad=fake, tokens=10)
    arr = (L.MemlayerRead * 9)(*([rd] * 9))
    u = C.c_void_p(fake)
    assert lib.memlayer_fetched_row_grads(C.byref(cfg), None, 1, u, None, None, None, None, 0, None) == \
        L.ERR_BAD_POINTER
    assert lib.memlayer_fetched_row_grads(C.byref(cfg), arr, 0, u, None, None, None, None, 0, None) == \
        L.ERR_BAD_SHAPE
    assert lib.memlayer_fetched_row_grads(C.byref(cfg), arr, 9, u, None, None, None, None, 0, None) == \
        L.ERR_BAD_SHAPE
    assert lib.memlayer_fetched_row_grads(C.byref(_cfg(d_value=66)), arr, 1, u, None, None, None, None, 0,
                                          None) == L.ERR_UNSUPPORTED
    assert lib.memlayer_fetched_row_grads(C.byref(cfg), arr, 1, None, None, None, None, None, 0, None) == \
        L.ERR_BAD_POINTER
    # workspace missing
    assert lib.memlayer_fetched_row_grads(C.byref(cfg), arr, 1, u, None, None, None, None, 0, None) == \
        L.ERR_WORKSPACE
    big = L.MemlayerRead(slots=fake, weights=fake, grad=fake, tokens=1 << 30)
    assert lib.memlayer_fetched_row_grads(C.byref(cfg), (L.MemlayerRead * 1)(big), 1, u, None, None, None,
                                          None, 0, None) == L.ERR_BAD_SHAPE
    ada = L.MemlayerAdagradArgs(values=fake, accum=fake, lr=0.1, grad_clip=1.0)
    assert lib.memlayer_row_adagrad(C.byref(_cfg(values_dtype=L.BF16)), arr, 1, C.byref(ada), None, 0, None) == \
        L.ERR_UNSUPPORTED
    assert lib.memlayer_row_adagrad(C.byref(cfg), arr, 1, None, None, 0, None) == L.ERR_BAD_POINTER
    assert lib.memlayer_row_adagrad(C.byref(cfg), arr, 1, C.byref(ada), None, 0, None) == L.ERR_WORKSPACE


def test_oracle_multi_read_merge_equals_dense_scatter():
    """Merging several layers' fetches (train.py:155-161 concatenation) is
    the dense scatter-add of every w * g into the table."""
    rng = np.random.default_rng(0)
    N, d = 64, 8
    parts, dense = [], np.zeros((N, d), np.float64)
    for M in (5, 9):
        s = rng.integers(0, N, (M, 2, 3))
        w = rng.random((M, 2, 3)).astype(np.float32)
        g = rng.standard_normal((M, d)).astype(np.float32)
        parts.append((s, w, g))
        for m in range(M):
            for h in range(2):
                for j in range(3):
                    dense[s[m, h, j]] += w[m, h, j] * g[m]
    sl = np.concatenate([p[0].reshape(-1) for p in parts])
    ww = np.concatenate([p[1].reshape(-1) for p in parts])
    gg = np.concatenate([np.repeat(p[2], 6, axis=0) for p in parts])
    uniq, rows = ref.fetched_row_grads(sl.reshape(-1, 1), ww.reshape(-1, 1), gg, N)
    np.testing.assert_array_equal(uniq, np.flatnonzero(np.abs(dense).sum(1) > 0))
    np.testing.assert_allclose(rows, dense[uniq], rtol=1e-5, atol=1e-6)
