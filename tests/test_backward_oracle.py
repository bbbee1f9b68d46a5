"""The oracle's backward through one memory layer (oracle layer_backward:
model.py:110-119 with memory.py:133-214, values excluded as with
sparse_grad) against float64 central differences of
sum(dy * y) + balance_coef * balance_loss with the routing held fixed (top-k
indices carry no gradient; f of the balance loss is a stop_gradient count).
The temperature sits inside its clamp range, where the straight-through
gradient is the plain one.  CPU only."""

import numpy as np
import pytest

from oracle import memlayer_ref as ref


def _setup(seed, query_scale=False, btgrad=False):
    cfg = ref.PoolConfig(n_sub_keys=8, heads=2, d_key=8, d_value=6, top_k=3, query_scale=query_scale,
                         balance_temperature_grad=btgrad, min_temperature=5.0, max_temperature=50.0)
    rng = np.random.default_rng(seed)
    T, dm = 5, 7
    p = {"h": rng.standard_normal((T, dm)), "w_router": rng.standard_normal((dm, 16)) * 0.5,
         "b_router": rng.standard_normal(16) * 0.1, "sub_keys": rng.standard_normal((2, 2, 8, 4)),
         "log_temperature": np.log(12.0), "w_gate": rng.standard_normal((dm, 6)) * 0.4,
         "b_gate": rng.standard_normal(6) * 0.1, "w_out": rng.standard_normal((6, dm)) * 0.4,
         "b_out": rng.standard_normal(dm) * 0.1}
    p = {k: np.asarray(v, np.float32) for k, v in p.items()}
    values = rng.standard_normal((64, 6)).astype(np.float32)
    dy = rng.standard_normal((T, dm))
    return cfg, p, values, dy


def _loss64(cfg, p, values, dy, fixed, bal, route_through_pool, probe=None, T_sg=None):
    """float64 forward with the base call's routing: sum(dy * y) + bal * balance_loss."""
    f = np.float64
    H, n, k, half = cfg.heads, cfg.n_sub_keys, cfg.top_k, cfg.d_key // 2
    h = np.asarray(p["h"], f)
    Tn = h.shape[0]
    q = (h @ p["w_router"].astype(f) + p["b_router"].astype(f)).reshape(Tn, H, 2, half)
    ss = np.sum(q * q, -1, keepdims=True) + 1e-6
    qn, q_len = q / np.sqrt(ss), np.sqrt(ss) / np.sqrt(half)
    x = p["sub_keys"].astype(f)
    kn = x / np.sqrt(np.sum(x * x, -1, keepdims=True) + 1e-6)
    lt = float(p["log_temperature"])
    T = np.exp(np.clip(lt, np.log(cfg.min_temperature), np.log(cfg.max_temperature)))
    cos = np.einsum("mhcd,hcnd->mhcn", qn, kn)
    scores = cos * T * (q_len if cfg.query_scale else 1.0)
    mi, hi = np.arange(Tn)[:, None, None], np.arange(H)[None, :, None]
    ss_ = scores[mi, hi, 0, fixed["idx_a"]] + scores[mi, hi, 1, fixed["idx_b"]]
    w = np.exp(ss_ - ss_.max(-1, keepdims=True))
    w /= w.sum(-1, keepdims=True)
    mem = np.einsum("mhk,mhkd->md", w, values.astype(f)[fixed["slots"]])
    if probe is not None:
        mem = mem + probe
    hg = np.asarray(p["h"], f) if not route_through_pool else np.asarray(fixed["h0"], f)
    zg = hg @ p["w_gate"].astype(f) + p["b_gate"].astype(f)
    gate = zg / (1 + np.exp(-zg))
    y = (mem * gate) @ p["w_out"].astype(f) + p["b_out"].astype(f)
    L = np.sum(dy * y)
    if bal:
        pp = scores if cfg.balance_temperature_grad else cos * T_sg
        sm = np.exp(pp - pp.max(-1, keepdims=True))
        sm /= sm.sum(-1, keepdims=True)
        P = sm.mean(0)
        L += bal * n * np.mean(np.sum(fixed["f"] * P, -1))
    return L


@pytest.mark.parametrize("query_scale,btgrad,bal,rtp", [(False, False, 0.0, False), (False, False, 0.7, False),
                                                        (True, False, 0.7, False), (False, True, 0.7, False),
                                                        (True, True, 0.3, True)])
def test_layer_backward_matches_central_differences(query_scale, btgrad, bal, rtp):
    cfg, p, values, dy = _setup(1, query_scale, btgrad)
    g = ref.layer_backward(cfg, p["h"], p["w_router"], p["b_router"], p["sub_keys"], p["log_temperature"], values,
                           p["w_gate"], p["b_gate"], p["w_out"], p["b_out"], dy, balance_coef=bal,
                           route_through_pool=rtp)
    q_raw = ref.dense(p["h"], p["w_router"], p["b_router"]).reshape(5, 2, 8)
    r = ref.route(cfg, q_raw, p["sub_keys"], p["log_temperature"])
    st = ref.pool_stats(cfg, r, False)
    fixed = dict(idx_a=r["idx_a"], idx_b=r["idx_b"], slots=r["slots"], f=st["balance_f"].astype(np.float64),
                 h0=p["h"])
    T_sg = float(r["temperature"])
    base = {k: v.astype(np.float64) if isinstance(v, np.ndarray) else float(v) for k, v in p.items()}
    eps = 1e-6
    rng = np.random.default_rng(7)
    for name in ("h", "w_router", "b_router", "sub_keys", "log_temperature", "w_gate", "b_gate", "w_out", "b_out"):
        val = base[name]
        if np.ndim(val) == 0:
            idxs = [()]
        else:
            flat = rng.choice(np.size(val), size=min(12, np.size(val)), replace=False)
            idxs = [np.unravel_index(i, np.shape(val)) for i in flat]
        for ix in idxs:
            pp, pm = dict(base), dict(base)
            if np.ndim(val) == 0:
                pp[name], pm[name] = val + eps, val - eps
            else:
                a, b = val.copy(), val.copy()
                a[ix] += eps
                b[ix] -= eps
                pp[name], pm[name] = a, b
            num = (_loss64(cfg, pp, values, dy, fixed, bal, rtp, T_sg=T_sg)
                   - _loss64(cfg, pm, values, dy, fixed, bal, rtp, T_sg=T_sg)) / (2 * eps)
            got = float(np.asarray(g[name])[ix])
            assert abs(got - num) <= 1e-4 * max(1.0, abs(num)), (name, ix, got, num)
    # the read-output (probe) gradient
    probe = np.zeros((5, 6))
    for ix in [(0, 0), (2, 3), (4, 5)]:
        a, b = probe.copy(), probe.copy()
        a[ix] += eps
        b[ix] -= eps
        num = (_loss64(cfg, base, values, dy, fixed, bal, rtp, probe=a, T_sg=T_sg)
               - _loss64(cfg, base, values, dy, fixed, bal, rtp, probe=b, T_sg=T_sg)) / (2 * eps)
        assert abs(g["probe"][ix] - num) <= 1e-4 * max(1.0, abs(num))


def test_probe_gradient_feeds_the_row_update():
    # the row gradients of the value table are sum over fetches of w * probe
    # (train.py:146-172); with the values differentiable that is d loss / d V
    cfg, p, values, dy = _setup(2)
    g = ref.layer_backward(cfg, p["h"], p["w_router"], p["b_router"], p["sub_keys"], p["log_temperature"], values,
                           p["w_gate"], p["b_gate"], p["w_out"], p["b_out"], dy)
    uniq, rows = ref.fetched_row_grads(g["slots"], g["weights"], g["probe"].astype(np.float32), cfg.pool_size)
    dense = np.zeros((cfg.pool_size, cfg.d_value))
    np.add.at(dense, g["slots"].reshape(-1), (g["weights"][..., None].astype(np.float64)
                                               * g["probe"][:, None, None, :]).reshape(-1, cfg.d_value))
    np.testing.assert_allclose(rows, dense[uniq], rtol=1e-5, atol=1e-6)


def _grads(cfg, p, values, dy, bal=0.0):
    return ref.layer_backward(cfg, p["h"], p["w_router"], p["b_router"], p["sub_keys"], p["log_temperature"],
                              values, p["w_gate"], p["b_gate"], p["w_out"], p["b_out"], dy, balance_coef=bal)


def test_clamped_temperature_passes_gradient_and_balance_reaches_it_only_when_asked():
    """test_memory_pool.py:79-101, gradient half: a temperature clamped at
    its floor still gets the read loss's gradient (straight-through,
    memory.py:141-146: d T / d log_t = the clamped T), and the balance loss
    moves the temperature only under balance_temperature_grad."""
    cfg, p, values, dy = _setup(3)                            # floor 5
    clamped = dict(p, log_temperature=np.float32(np.log(2.0)))
    at_floor = dict(p, log_temperature=np.float32(np.log(5.0)))
    g_c, g_f = _grads(cfg, clamped, values, dy), _grads(cfg, at_floor, values, dy)
    assert g_c["log_temperature"] != 0.0
    assert np.array_equal(g_c["slots"], g_f["slots"])
    np.testing.assert_allclose(g_c["log_temperature"], g_f["log_temperature"], rtol=1e-6)
    zero = np.zeros_like(dy)
    for btgrad in (False, True):
        cfg_b, p_b, values_b, _ = _setup(3, btgrad=btgrad)
        g_b = _grads(cfg_b, p_b, values_b, zero, bal=1.0)
        if btgrad:
            assert g_b["log_temperature"] != 0.0
        else:
            assert g_b["log_temperature"] == 0.0
            assert np.abs(g_b["sub_keys"]).max() > 0.0          # the balance term still reaches the keys
