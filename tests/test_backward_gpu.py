"""GPU parity of the memory-layer backward (memlayer_layer_backward) against
the oracle's layer_backward (model.py:110-119 with memory.py:133-214, values
excluded as with sparse_grad), through MemoryLayer.apply_train / backward.

Each gradient must match within 1e-4 of its largest entry (float32 sums in
fixed orders against the oracle's float64); the forward's slots are first
checked equal to the oracle's (the gradients follow the routing)."""

import numpy as np
import pytest
import torch

from model_b200 import MemoryLayer, MemoryPool
from oracle import memlayer_ref as ref

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _case(n, H, dk, d, k, dm, M, seed, vdt=torch.float32, query_scale=False, btgrad=False, cpu_rng=False):
    # cpu_rng: biases, h and dy drawn on the host, so that a case's routing
    # margins can be checked beforehand without a GPU
    pool = MemoryPool(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k, query_scale=query_scale,
                      balance_temperature_grad=btgrad, min_temperature=5.0, max_temperature=50.0)
    layer = MemoryLayer(pool, d_model=dm, layer=1)
    params = layer.init(seed, values_dtype=vdt)
    dev = "cpu" if cpu_rng else "cuda"
    with torch.no_grad():
        params["pool"]["log_temperature"].fill_(float(np.log(12.0)))
        g = torch.Generator("cpu").manual_seed(seed)
        for name in ("router_1", "mem_gate_1", "mem_out_1"):
            if cpu_rng:
                params[name]["bias"].copy_(torch.empty(params[name]["bias"].shape).normal_(0.0, 0.1, generator=g))
            else:
                params[name]["bias"].normal_(0.0, 0.1, generator=torch.Generator("cuda").manual_seed(seed))
    h = torch.randn(M, dm, device=dev, generator=torch.Generator(dev).manual_seed(seed + 1)).to("cuda")
    dy = torch.randn(M, dm, device=dev, generator=torch.Generator(dev).manual_seed(seed + 2)).to("cuda")
    cfg = ref.PoolConfig(n_sub_keys=n, heads=H, d_key=dk, d_value=d, top_k=k, query_scale=query_scale,
                         balance_temperature_grad=btgrad, min_temperature=5.0, max_temperature=50.0)
    return layer, params, h, dy, cfg


def _np(t):
    return t.detach().float().cpu().numpy()


def _check(layer, params, h, dy, cfg, bal, rtp=False, gumbel=None, drop_mem=False):
    train = gumbel is not None
    y, mem, aux, ctx = layer.apply_train(params, h, train=train, gumbel=gumbel, check=True)
    if drop_mem:   # a caller that kept no read output: the backward re-gathers it
        ctx["la"].mem = None
    g = layer.backward(ctx, dy, balance_coef=bal, route_through_pool=rtp, check=True)
    torch.cuda.synchronize()
    p = params
    want = ref.layer_backward(cfg, _np(h), _np(p["router_1"]["kernel"]), _np(p["router_1"]["bias"]),
                              _np(p["pool"]["sub_keys"]), float(p["pool"]["log_temperature"]),
                              _np(p["pool"]["values"]), _np(p["mem_gate_1"]["kernel"]), _np(p["mem_gate_1"]["bias"]),
                              _np(p["mem_out_1"]["kernel"]), _np(p["mem_out_1"]["bias"]), _np(dy),
                              balance_coef=bal, route_through_pool=rtp, train=train,
                              gumbel=None if gumbel is None else _np(gumbel))
    assert np.array_equal(_np(aux["slots"]).astype(np.int64), want["slots"]), "forward routing differs from the oracle"
    got = {"h": g["h"], "w_router": g["router_1"]["kernel"], "b_router": g["router_1"]["bias"],
           "sub_keys": g["pool"]["sub_keys"], "log_temperature": g["pool"]["log_temperature"],
           "w_gate": g["mem_gate_1"]["kernel"], "b_gate": g["mem_gate_1"]["bias"],
           "w_out": g["mem_out_1"]["kernel"], "b_out": g["mem_out_1"]["bias"], "probe": g["probe"]}
    for name, t in got.items():
        a, b = _np(t).reshape(-1), np.asarray(want[name], np.float64).reshape(-1)
        scale = max(np.abs(b).max(), 1e-12)
        err = np.abs(a - b).max() / scale
        assert err <= TOL, f"{name}: {err:.2e} of max |grad| {scale:.3e}"


@pytest.mark.parametrize("bal", [0.0, 0.7])
@pytest.mark.parametrize("query_scale", [False, True])
def test_backward_matches_oracle_small(bal, query_scale):
    _check(*_case(32, 2, 32, 32, 8, 48, 100, seed=3, query_scale=query_scale), bal)


def test_backward_temperature_grad_and_route_through_pool():
    _check(*_case(32, 2, 32, 32, 8, 48, 100, seed=4, query_scale=True, btgrad=True), 0.3, rtp=True)


def test_backward_half_table_and_noisy_forward():
    layer, params, h, dy, cfg = _case(48, 2, 32, 64, 8, 32, 77, seed=5, vdt=torch.float16)
    gumbel = -torch.log(-torch.log(torch.rand(77, 2, 2, 48, device="cuda",
                                              generator=torch.Generator("cuda").manual_seed(9)).clamp_(min=1e-12)))
    _check(layer, params, h, dy, cfg, 0.5, gumbel=gumbel)


def test_backward_cfg0_shapes():
    # configs[0] shapes at 512 tokens: H 4, n 512, d_key 256, d 256, k 16, d_model 256
    _check(*_case(512, 4, 256, 256, 16, 256, 512, seed=6), 0.01)


@pytest.mark.parametrize("n,H,dk,M,qs,bt,bal", [
    (128, 1, 64, 2100, True, True, 0.8),      # half 32; 17 token tiles, the last partial; K slices of d k_hat
    (256, 2, 128, 300, False, False, 0.6),    # half 64; a partial last tile
    (512, 2, 256, 640, True, False, 1.0),     # half 128: the d q_hat accumulator spans 4 cosine chunks
])
def test_backward_balance_on_tensor_cores(n, H, dk, M, qs, bt, bal):
    # sub-key counts that are multiples of 128 (up to 512) take the fused
    # cosine -> softmax -> d cos kernel; a strong balance coefficient makes
    # its share of every gradient visible
    _check(*_case(n, H, dk, 64, 8, 64, M, seed=7 + n, query_scale=qs, btgrad=bt), bal)


@pytest.mark.parametrize("n,H,dk,M,qs,bt,bal,seed", [
    (128, 1, 256, 129, False, True, 0.9, 116),   # half 128 = n: d q_hat overwrites every cosine column; one token in the last tile
    (384, 2, 64, 300, True, False, 0.7, 102),    # three 128-key blocks per K stage, twelve 32-key chunks
])
def test_backward_balance_on_tensor_cores_edge_shapes(n, H, dk, M, qs, bt, bal, seed):
    # host-drawn inputs whose routing margins (the gap after the k-th score
    # of each half and after the k-th of the k x k candidates) exceed 1e-4
    _check(*_case(n, H, dk, 64, 8, 64, M, seed=seed, query_scale=qs, btgrad=bt, cpu_rng=True), bal)


def test_backward_balance_on_tensor_cores_noisy_forward():
    # selection noise: the routing backward takes each selected sub-key's
    # cosine from the forward's clean scores (not its noisy selection scores)
    layer, params, h, dy, cfg = _case(128, 2, 64, 64, 8, 64, 300, seed=21, query_scale=True)
    gumbel = -torch.log(-torch.log(torch.rand(300, 2, 2, 128, device="cuda",
                                              generator=torch.Generator("cuda").manual_seed(22)).clamp_(min=1e-12)))
    _check(layer, params, h, dy, cfg, 0.5, gumbel=gumbel)


@pytest.mark.parametrize("n,H,dk,d,dm,M", [
    (32, 2, 32, 48, 40, 333),     # K tails (333 tokens, d_model 40), 48- and 64-column tiles
    (32, 2, 32, 48, 50, 260),     # d_model 50: a row pitch the bulk copies cannot take (fallback GEMM)
    (64, 3, 64, 80, 96, 200),     # 3 heads: 192 router columns
])
def test_backward_odd_shapes(n, H, dk, d, dm, M):
    _check(*_case(n, H, dk, d, 8, dm, M, seed=50 + dm), 0.4)


@pytest.mark.parametrize("vdt", [torch.float32, torch.float16])
def test_backward_without_forward_read_output(vdt):
    # the configs[0] case's seed (its routing has no near-ties against the oracle)
    _check(*_case(512, 4, 256, 256, 16, 256, 512, seed=6, vdt=vdt), 0.05, drop_mem=True)


def test_backward_no_tokens():
    layer, params, h, dy, _ = _case(32, 2, 32, 32, 8, 48, 100, seed=6)
    y, mem, aux, ctx = layer.apply_train(params, h[:0], check=True)
    assert y.shape == (0, 48) and mem.shape == (0, 32) and aux["slots"].shape == (0, 2, 8)
    g = layer.backward(ctx, dy[:0], balance_coef=0.5, check=True)
    torch.cuda.synchronize()
    assert g["h"].shape == (0, 48) and g["probe"].shape == (0, 32)
    for name in ("router_1", "mem_gate_1", "mem_out_1"):
        for leaf in ("kernel", "bias"):
            assert not g[name][leaf].any(), f"{name}/{leaf} not zero for no tokens"
    assert not g["pool"]["sub_keys"].any() and float(g["pool"]["log_temperature"]) == 0.0
