"""The backbone oracle (oracle/backbone_ref.py) on the CPU: the reference's
own property that decoding with the cache reproduces the full forward
(tests/test_memory_pool.py:486-502, atol 1e-4), causality, and known answers
of the restated flax layers (LayerNorm with its fast variance, the tanh
GELU)."""

import numpy as np
import pytest

from oracle import backbone_ref as br
from oracle import memlayer_ref as ml


def _cfg(**kw):
    P = ml.PoolConfig(n_sub_keys=16, heads=2, d_key=16, d_value=24, top_k=4)
    base = dict(vocab_size=50, max_len=12, d_model=32, n_layers=3, n_heads=4, ffn_mult=2, memory_layers=(1,), pool=P)
    base.update(kw)
    return br.ModelCfg(**base)


@pytest.mark.parametrize("memory_ffn", [False, True])
def test_decode_with_cache_equals_full_forward(memory_ffn):
    cfg = _cfg(memory_ffn=memory_ffn)
    p = br.init_params(cfg, 0)
    tok = np.random.default_rng(1).integers(0, 50, (2, 10))
    full = br.forward(cfg, p, tok)
    cache = br.empty_cache(cfg, 2)
    steps = np.stack([br.decode_step(cfg, p, cache, tok[:, t], t) for t in range(10)], 1)
    np.testing.assert_allclose(steps, full, atol=1e-4)


def test_forward_is_causal():
    cfg = _cfg()
    p = br.init_params(cfg, 2)
    tok = np.random.default_rng(3).integers(0, 50, (1, 10))
    a = br.forward(cfg, p, tok)
    tok2 = tok.copy()
    tok2[0, 6:] = (tok2[0, 6:] + 7) % 50
    b = br.forward(cfg, p, tok2)
    np.testing.assert_array_equal(a[0, :6], b[0, :6])
    assert np.abs(a[0, 6:] - b[0, 6:]).max() > 0


def test_layer_norm_known_answers():
    x = np.array([[1.0, 2.0, 3.0, 4.0], [5.0, 5.0, 5.0, 5.0]], np.float32)
    y = br.layer_norm(x, np.ones(4, np.float32), np.zeros(4, np.float32))
    # mean 2.5, variance 1.25 (E[x^2] - E[x]^2 = 7.5 - 6.25)
    np.testing.assert_allclose(y[0], (x[0] - 2.5) / np.sqrt(1.25 + 1e-6), rtol=1e-6)
    np.testing.assert_array_equal(y[1], np.zeros(4, np.float32))        # zero variance: x - mean = 0
    y2 = br.layer_norm(x, np.full(4, 2.0, np.float32), np.full(4, 0.5, np.float32))
    np.testing.assert_allclose(y2, 2.0 * y + 0.5, rtol=1e-6)


def test_gelu_tanh_form_known_answers():
    g = br.gelu(np.array([0.0, 1.0, -1.0, 3.0], np.float32))
    want = [0.0, 0.8411920, -0.1588080, 2.9963627]                       # 0.5x(1+tanh(sqrt(2/pi)(x+0.044715x^3)))
    np.testing.assert_allclose(g, want, rtol=1e-5, atol=1e-7)


def test_generate_greedy_continues_with_argmax():
    cfg = _cfg()
    p = br.init_params(cfg, 4)
    prompt = np.random.default_rng(5).integers(0, 50, (2, 3))
    out = br.generate(cfg, p, prompt, 4)
    assert out["tokens"].shape == (2, 4) and out["logits"].shape == (2, 6, 50)
    np.testing.assert_array_equal(out["tokens"], np.argmax(out["logits"][:, 2:], -1))
    with pytest.raises(ValueError):
        br.generate(cfg, p, prompt, 10)
