"""Calls issued on a side stream (``stream=``) give the same results as on
the current stream, and the blocks they allocate stay theirs while their
kernels run: right after each side-stream call returns, the current stream
allocates and overwrites fresh memory before the side stream is waited for."""

import pytest
import torch

from model_b200 import MemoryLayer, MemoryPool
from model_b200 import keys as K
from model_b200 import sparse as S

pytestmark = pytest.mark.gpu


def _scribble():
    # the allocator would hand these blocks out first if a side-stream call
    # had released its workspace back to the current stream
    for mb in (1, 4, 16, 64):
        torch.empty(mb << 18, device="cuda").fill_(float("nan"))


def _layer(seed=7):
    pool = MemoryPool(n_sub_keys=64, heads=2, d_key=32, d_value=64, top_k=8, min_temperature=5.0)
    layer = MemoryLayer(pool, d_model=48, layer=1)
    params = layer.init(seed)
    h = torch.randn(300, 48, device="cuda", generator=torch.Generator("cuda").manual_seed(seed))
    dy = torch.randn(300, 48, device="cuda", generator=torch.Generator("cuda").manual_seed(seed + 1))
    return layer, params, h, dy


def test_layer_forward_and_backward_on_side_stream():
    layer, params, h, dy = _layer()
    y0, mem0, aux0, ctx0 = layer.apply_train(params, h, check=True)
    g0 = layer.backward(ctx0, dy, balance_coef=0.3, check=True)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    y1, mem1, aux1, ctx1 = layer.apply_train(params, h, stream=side)
    g1 = layer.backward(ctx1, dy, balance_coef=0.3, stream=side)
    _scribble()
    side.synchronize()
    torch.cuda.synchronize()
    assert torch.equal(y0, y1) and torch.equal(mem0, mem1)
    assert torch.equal(aux0["slots"], aux1["slots"])
    # every sum of the backward runs in a fixed order on the library's own
    # kernels: the same gradients bit for bit on any stream
    for a, b in ((g0["h"], g1["h"]), (g0["router_1"]["kernel"], g1["router_1"]["kernel"]),
                 (g0["pool"]["sub_keys"], g1["pool"]["sub_keys"]), (g0["probe"], g1["probe"])):
        assert torch.equal(a, b)


def test_two_backward_calls_overlapping_on_two_streams():
    # no shared GEMM state: two backward calls may run at the same time on one
    # device (128 sub-keys: the balance term takes the fused tensor-core kernel)
    pool = MemoryPool(n_sub_keys=128, heads=2, d_key=64, d_value=64, top_k=8, min_temperature=5.0)
    layer = MemoryLayer(pool, d_model=64, layer=1)
    params = layer.init(5)
    h = torch.randn(600, 64, device="cuda", generator=torch.Generator("cuda").manual_seed(5))
    dy = torch.randn(600, 64, device="cuda", generator=torch.Generator("cuda").manual_seed(6))
    y0, mem0, aux0, ctx0 = layer.apply_train(params, h, check=True)
    g0 = layer.backward(ctx0, dy, balance_coef=0.3, check=True)
    torch.cuda.synchronize()
    ctxs = [layer.apply_train(params, h)[3] for _ in range(2)]
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    gs = [layer.backward(c, dy, balance_coef=0.3, stream=st) for c, st in zip(ctxs, streams)]
    for st in streams:
        st.synchronize()
    for g in gs:
        for name in ("h", "probe"):
            assert torch.equal(g0[name], g[name]), name
        for name in ("router_1", "mem_gate_1", "mem_out_1"):
            assert torch.equal(g0[name]["kernel"], g[name]["kernel"]) and torch.equal(g0[name]["bias"], g[name]["bias"])
        assert torch.equal(g0["pool"]["sub_keys"], g["pool"]["sub_keys"])


def test_pool_keys_and_row_update_on_side_stream():
    layer, params, h, _ = _layer(11)
    P, pp = layer.pool, params["pool"]
    q = torch.randn(300, P.heads, P.d_key, device="cuda", generator=torch.Generator("cuda").manual_seed(3))
    out0, aux0 = P.apply({"params": pp}, q)
    loss0, kg0 = K.key_diversity_loss(pp["sub_keys"], grad=True)
    probe = torch.randn(300, P.d_value, device="cuda", generator=torch.Generator("cuda").manual_seed(4))
    v0, a0 = pp["values"].clone(), torch.zeros(P.pool_size, device="cuda")
    r0 = S.rowwise_adagrad(v0, a0, {"slots": [aux0["slots"]], "weights": [aux0["weights"]]}, {1: probe}, [1],
                           lr=0.1, grad_clip=1.0)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    out1, aux1 = P.apply({"params": pp}, q, stream=side)
    loss1, kg1 = K.key_diversity_loss(pp["sub_keys"], grad=True, stream=side)
    v1, a1 = pp["values"].clone(), torch.zeros(P.pool_size, device="cuda")
    side.wait_stream(torch.cuda.current_stream())
    r1 = S.rowwise_adagrad(v1, a1, {"slots": [aux1["slots"]], "weights": [aux1["weights"]]}, {1: probe}, [1],
                           lr=0.1, grad_clip=1.0, stream=side)
    _scribble()
    side.synchronize()
    torch.cuda.synchronize()
    assert torch.equal(out0, out1) and torch.equal(aux0["slots"], aux1["slots"])
    assert torch.equal(loss0, loss1) and torch.equal(kg0, kg1)
    assert torch.equal(v0, v1) and torch.equal(a0, a1)
    assert torch.equal(r0["clip_scale"], r1["clip_scale"]) and torch.equal(r0["n_unique"], r1["n_unique"])
