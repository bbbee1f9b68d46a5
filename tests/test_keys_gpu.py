"""GPU parity of the sub-key maintenance kernels (memory.py:230-281)
against the CPU oracle, through the C ABI.

Tolerances: the diversity loss is ||K^T K||_F^2 - sum |k|^4 on the GPU and a
direct sum of squared off-diagonal cosines in the oracle, so it is compared
within 1e-5 of the magnitude of the cancelled terms (loss + n / (n - 1) per
codebook); gradients within 1e-4 of their largest magnitude (float32 sums
of n terms in different orders).  Revival: the dead mask and untouched keys
are bit-exact; revived keys and usage within 1e-6 relative."""

import numpy as np
import pytest
import torch

from model_b200 import keys as K
from oracle import memlayer_ref as ref

pytestmark = pytest.mark.gpu


def _keys(H, n, half, seed, clumped=False):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((H, 2, n, half)).astype(np.float32)
    if clumped:   # keys that crowd one region (large off-diagonal cosines)
        x += 3.0 * rng.standard_normal((H, 2, 1, half)).astype(np.float32)
    return x * rng.uniform(0.5, 2.0, (H, 2, n, 1)).astype(np.float32)


@pytest.mark.parametrize("H,n,half,clumped", [(2, 8, 4, False), (3, 37, 20, True), (4, 512, 128, False),
                                              (8, 1024, 64, True), (4, 64, 128, False)])
def test_key_diversity_matches_oracle(H, n, half, clumped):
    x = _keys(H, n, half, seed=n + half, clumped=clumped)
    want_loss, want_grad = ref.key_diversity_loss(x)
    xt = torch.from_numpy(x).cuda()
    loss, grad = K.key_diversity_loss(xt, grad=True, grad_scale=0.01)
    loss_only = K.key_diversity_loss(xt)
    torch.cuda.synchronize()
    scale = float(want_loss) + n / (n - 1.0)
    assert abs(float(loss) - float(want_loss)) <= 1e-5 * scale
    assert float(loss_only) == float(loss)
    g = grad.cpu().numpy()
    assert np.abs(g - 0.01 * want_grad).max() <= 1e-4 * 0.01 * np.abs(want_grad).max()


def test_key_diversity_known_answers():
    # the reference's test uses one codebook ([1, 1, 4, 4]); the pool's
    # sub_keys hold two per head, and the loss is a mean over codebooks
    eye = torch.eye(4, device="cuda")[None, None].expand(1, 2, 4, 4)
    assert abs(float(K.key_diversity_loss(eye))) <= 1e-6
    same = torch.ones(1, 2, 4, 4, device="cuda")
    assert float(K.key_diversity_loss(same)) == pytest.approx(1.0, abs=1e-4)
    one = torch.randn(2, 2, 1, 8, device="cuda")        # n = 1: 0 / 0 as in the reference
    assert torch.isnan(K.key_diversity_loss(one))


def test_key_diversity_is_deterministic():
    x = torch.from_numpy(_keys(4, 512, 128, seed=3, clumped=True)).cuda()
    a = K.key_diversity_loss(x, grad=True)
    b = K.key_diversity_loss(x, grad=True)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.parametrize("H,n,half,M,threshold,noise", [(2, 8, 4, 32, 0.1, 0.0), (2, 8, 4, 32, 0.5, 0.05),
                                                       (4, 512, 128, 1000, 0.5, 0.05),
                                                       (8, 1024, 64, 4096, 0.8, 0.05), (3, 37, 20, 7, 0.9, 0.2)])
def test_revive_matches_oracle(H, n, half, M, threshold, noise):
    rng = np.random.default_rng(n + M)
    keys = ref.l2_normalize(rng.standard_normal((H, 2, n, half)).astype(np.float32))
    usage = rng.dirichlet(np.full(n, 0.3), (H, 2)).astype(np.float32)
    queries = ref.l2_normalize(rng.standard_normal((M, H, 2, half)).astype(np.float32))
    pick = rng.integers(0, M, (H, 2, n)).astype(np.int32)
    normal = rng.standard_normal((H, 2, n, half)).astype(np.float32)
    want_k, want_u, want_d = ref.revive_dead_keys(keys, usage, queries, pick, normal, threshold, noise_scale=noise)
    assert want_d.any()
    m0 = torch.full((H, 2, n, half), 3.0, device="cuda")
    m1 = torch.full((H, 2, n, half), 5.0, device="cuda")
    got_k, got_u, got_d = K.revive_dead_keys(torch.from_numpy(keys).cuda(), torch.from_numpy(usage).cuda(),
                                             torch.from_numpy(queries).cuda(), threshold, noise,
                                             pick=torch.from_numpy(pick).cuda(),
                                             normal=torch.from_numpy(normal).cuda(), moments=(m0, m1))
    torch.cuda.synchronize()
    got_d = got_d.cpu().numpy()
    np.testing.assert_array_equal(got_d, want_d)
    gk = got_k.cpu().numpy()
    np.testing.assert_array_equal(gk[~want_d], keys[~want_d])
    np.testing.assert_allclose(gk[want_d], want_k[want_d], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(got_u.cpu().numpy(), want_u, rtol=1e-6, atol=1e-9)
    for m, v in ((m0, 3.0), (m1, 5.0)):
        m = m.cpu().numpy()
        assert (m[want_d] == 0).all() and (m[~want_d] == v).all()


def test_revive_with_device_draws_keeps_a_distribution():
    H, n, half = 2, 64, 16
    g = torch.Generator("cuda").manual_seed(0)
    keys = torch.nn.functional.normalize(torch.randn(H, 2, n, half, device="cuda"), dim=-1)
    usage = torch.distributions.Dirichlet(torch.full((n,), 0.3)).sample((H, 2)).cuda()
    queries = torch.nn.functional.normalize(torch.randn(50, H, 2, half, device="cuda"), dim=-1)
    new_k, new_u, dead = K.revive_dead_keys(keys, usage, queries, 0.5, generator=g)
    assert int(dead.sum()) > 0
    torch.testing.assert_close(new_u.sum(-1), torch.ones(H, 2, device="cuda"), rtol=1e-5, atol=0)
    torch.testing.assert_close(new_k.norm(dim=-1), torch.ones(H, 2, n, device="cuda"), rtol=1e-5, atol=1e-5)
    assert torch.equal(new_k[~dead], keys[~dead])
