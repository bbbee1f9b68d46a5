"""Decode steps as CUDA graphs (memory_pool_model/generate.py:23-34 step):
LayerDecodeStep's graph replays must give exactly the outputs of
MemoryLayer.apply on the same hidden states, step after step with new
inputs, at decode batch sizes (batch 200 takes the tensor-core projection
path)."""

import pytest
import torch

from model_b200 import MemoryLayer, MemoryPool
from model_b200.generate import LayerDecodeStep

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("batch", [1, 8, 64, 200])
@pytest.mark.parametrize("vdt", [torch.float32, torch.float16])
def test_graph_steps_match_eager_layer(batch, vdt):
    pool = MemoryPool(n_sub_keys=256, heads=4, d_key=128, d_value=256, top_k=16)
    layer = MemoryLayer(pool, d_model=256, layer=1)
    params = layer.init(0, values_dtype=vdt)
    step = LayerDecodeStep(layer, params, batch)
    eager = LayerDecodeStep(layer, params, batch, graph=False)
    g = torch.Generator("cuda").manual_seed(batch)
    prev = None
    for i in range(4):
        h = torch.randn(batch, 256, device="cuda", generator=g)
        y, mem, aux = step.step(h)
        y0, mem0, aux0 = layer.apply(params, h, check=True)
        ye, meme, auxe = eager.step(h)
        torch.cuda.synchronize()
        assert torch.equal(y, y0) and torch.equal(mem, mem0)
        assert torch.equal(aux["slots"], aux0["slots"]) and torch.equal(aux["weights"], aux0["weights"])
        assert torch.equal(ye, y0) and torch.equal(auxe["slots"], aux0["slots"])
        if prev is not None:
            assert not torch.equal(y, prev)          # the replay read the new inputs
        prev = y.clone()
    assert step.status() == 0 and eager.status() == 0


def test_graph_step_rejects_wrong_batch():
    pool = MemoryPool(n_sub_keys=64, heads=2, d_key=32, d_value=32, top_k=4)
    layer = MemoryLayer(pool, d_model=32, layer=1)
    step = LayerDecodeStep(layer, layer.init(0), 4)
    with pytest.raises(ValueError):
        step.step(torch.zeros(5, 32, device="cuda"))


def test_refresh_after_weight_update():
    pool = MemoryPool(n_sub_keys=128, heads=2, d_key=64, d_value=64, top_k=8)
    layer = MemoryLayer(pool, d_model=64, layer=1)
    params = layer.init(0)
    step = LayerDecodeStep(layer, params, 8)
    h = torch.randn(8, 64, device="cuda", generator=torch.Generator("cuda").manual_seed(3))
    with torch.no_grad():                         # an in-place weight update
        params["pool"]["sub_keys"].mul_(-1.0)
        params["router_1"]["kernel"].add_(0.5)
    step.refresh()
    y, _, aux = step.step(h)
    y0, _, aux0 = layer.apply(params, h)
    torch.cuda.synchronize()
    assert torch.equal(y, y0) and torch.equal(aux["slots"], aux0["slots"])
